/*
 * ptxgen_b200.h - the C ABI of the B200 launcher for ptxgen-emitted PTX.
 *
 * The reference compiler (alexpejovic/emmy-hackathon-submission, a Python package) stops at PTX
 * text: `python compile.py <k>.ir.json > k.ptx` (reference compile.py:58-69). Its evaluator
 * (emmy-hackathon-2026/submit.py, an un-vendored submodule) loaded that PTX and launched it
 * through the CUDA driver with the launch contract of meta.json (reference
 * tools/generate.py:99-107): a 1-D grid of meta.grid[0] blocks of meta.block[0] threads,
 * meta.smem_bytes of dynamic shared memory, one device pointer per meta.arg_order entry, and
 * the meta.zero_outputs buffers zeroed before the launch. Each entry point below is one step of
 * that launch, so a caller binds exactly what the evaluator did:
 *
 *   pg_init            <- the driver/context set-up of the evaluator
 *   pg_module_load     <- cuModuleLoadData of the compiler's stdout, with the JIT log kept
 *   pg_kernel_get      <- cuModuleGetFunction(meta.kernels[i].entry)
 *   pg_kernel_launch   <- cuLaunchKernel(grid, block, smem, args in meta.arg_order)
 *   pg_memset_async    <- zeroing meta.zero_outputs (tools/generate.py:106)
 *   pg_run_host        <- the whole evaluator step on host buffers: copy in, zero, launch,
 *                         copy out, check the kernel's status word
 *
 * pg_kernel_time is the timing the evaluator did around its launches (warm-up launches, then
 * one CUDA event pair per timed launch), for callers that have no other timer.
 *
 * Some entry points have no counterpart in the reference, because its kernels never needed
 * them: pg_tensormap_fill writes a TMA tensor map into a module's .global symbol (the tcgen05
 * templates read their operands through TMA, and a kernel's parameters must stay the plain
 * device pointers of meta.arg_order), pg_status_take reads the status word that kernels with
 * bounded waits set instead of hanging, pg_kernel_max_clusters sizes the grid of a
 * persistent kernel whose CTAs run in pairs (the tcgen05 GEMM's 2-SM form), and
 * pg_ipc_handle/pg_ipc_open/pg_ipc_close map the buffers through which ranks on other GPUs
 * exchange partial results over NVLink (the reference runs on one GPU).
 *
 * Plain C types only: device pointers and CUDA streams travel as uint64_t. Every function
 * returns 0 on success, a positive CUresult from the driver, or a negative PG_ERR_* code;
 * pg_last_error() describes the last failure on the calling thread (including the PTX JIT
 * error log). No function allocates device memory.
 */
#ifndef PTXGEN_B200_H
#define PTXGEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PG_OK 0
#define PG_ERR_NO_DRIVER (-1)     /* libcuda.so.1 could not be loaded or lacks a symbol */
#define PG_ERR_ARGUMENT (-2)      /* a null handle, a bad size or an unknown enum value */
#define PG_ERR_NOT_FOUND (-3)     /* no such entry or .global symbol in the module */
#define PG_ERR_KERNEL_STATUS (-4) /* the kernel set its status word (a bounded wait gave up) */
#define PG_ERR_NOT_INITIALISED (-5)
#define PG_ERR_RUNTIME (-6)       /* a CUDA runtime call failed (pg_grid_sum_f32_noalloc) */

/* Element types of pg_tensormap_fill. */
#define PG_DT_U8 0
#define PG_DT_F16 1
#define PG_DT_BF16 2
#define PG_DT_F32 3

/* Flags of pg_run_host, per argument. */
#define PG_ARG_IN 1u   /* copy host -> device before the launch */
#define PG_ARG_ZERO 2u /* zero on the device before the launch */
#define PG_ARG_OUT 4u  /* copy device -> host after the launch */

typedef struct pg_module pg_module;
typedef struct pg_kernel pg_kernel;

/* Load libcuda, initialise the driver and make device `device`'s primary context current on
 * the calling thread (the context PyTorch's runtime uses, so its pointers are valid here). */
int pg_init(int device);

/* Describes the last failure on this thread; never NULL. */
const char *pg_last_error(void);

/* JIT-compile a NUL-terminated PTX module. On a JIT error the log is in pg_last_error(). */
int pg_module_load(const char *ptx, pg_module **out);
int pg_module_unload(pg_module *module);

/* The kernel named `entry` in `module`. */
int pg_kernel_get(pg_module *module, const char *entry, pg_kernel **out);

/* Launch with a 1-D grid; `ptrs[i]` is the device address of the i-th parameter (every
 * parameter of a ptxgen kernel is a .u64 device pointer). Dynamic shared memory above 48 KiB
 * is opted into automatically. Asynchronous on `stream` (0 = the legacy default stream). */
int pg_kernel_launch(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                     uint64_t stream, const uint64_t *ptrs, int nptrs);

/* pg_kernel_launch_ex flag: launch with programmatic stream serialization
 * (CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION). The kernel may then start while the
 * kernel before it on the stream still runs, once that kernel has executed
 * griddepcontrol.launch_dependents (or ended); it must execute griddepcontrol.wait before it
 * touches anything that kernel writes. ptxgen uses it for the split-K GEMM after the module's
 * own kernel that zeroes C (which the launcher launches plainly, so it follows all earlier
 * work): the GEMM's set-up and MMAs overlap the zeroing, and its epilogue waits before adding
 * into C. No counterpart in the reference, whose evaluator zeroes with a memset. */
#define PG_LAUNCH_EARLY 1u

/* pg_kernel_launch with `flags` (0 or PG_LAUNCH_EARLY; anything else is PG_ERR_ARGUMENT). */
int pg_kernel_launch_ex(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                        uint64_t stream, const uint64_t *ptrs, int nptrs, uint32_t flags);

/* Launch like pg_kernel_launch `warmup` times untimed, then `reps` times, each bracketed by
 * CUDA events on `stream`; waits for the last and writes launch i's device time in
 * milliseconds to ms_out[i]. Launches run back to back (no cache flush between them). */
int pg_kernel_time(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                   uint64_t stream, const uint64_t *ptrs, int nptrs, int warmup, int reps,
                   float *ms_out);

/* How many clusters of `cluster` CTAs of `block` threads and `smem_bytes` of dynamic shared
 * memory can be resident on the device at once (cuOccupancyMaxActiveClusters); a persistent
 * kernel compiled for that cluster size launches at most that many clusters. */
int pg_kernel_max_clusters(pg_kernel *kernel, uint32_t block, uint32_t smem_bytes,
                           uint32_t cluster, int *out);

/* Encode a tiled TMA tensor map (cuTensorMapEncodeTiled) over the row-major array at `base`
 * and write its 128 bytes into the module's .global symbol `symbol`. dims[0] is the innermost
 * extent in elements; strides_bytes[i] is the byte stride of dimension i+1 (rank-1 entries);
 * box[i] is the tile extent copied per load; swizzle_bytes is 0, 32, 64 or 128. A call with the
 * same arguments as the previous one for that symbol copies nothing. */
int pg_tensormap_fill(pg_module *module, const char *symbol, int dtype, int rank, uint64_t base,
                      const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                      int swizzle_bytes);

/* Copy `bytes` bytes from host memory into the module's .global symbol `symbol` (at most its
 * size). Synchronous. No counterpart in the reference: a kernel whose partial result is summed
 * across ranks inside the kernel reads its exchange configuration (peer addresses, rank) from
 * module globals, so its parameters stay the plain device pointers of meta.arg_order. */
int pg_global_write(pg_module *module, const char *symbol, const void *data, size_t bytes);

/* Read the module's 32-bit status word (.global ptxgen_status) into *status and clear it;
 * *status is 0 when the module has none. Synchronous. */
int pg_status_take(pg_module *module, uint32_t *status);

/* CUDA IPC over one device allocation, for buffers that other processes' kernels reach through
 * NVLink (ptxgen.peer's cross-rank sum). No counterpart in the reference, which runs on one
 * GPU. pg_ipc_handle writes the PG_IPC_HANDLE_BYTES-byte handle of the allocation holding `ptr`
 * and ptr's byte offset inside it; pg_ipc_open maps another process's allocation by its
 * handle, *base being its first byte here (peer access enabled as needed); pg_ipc_close
 * unmaps it. An allocation of this process cannot be opened here. */
#define PG_IPC_HANDLE_BYTES 64
int pg_ipc_handle(uint64_t ptr, void *handle, uint64_t *offset);
int pg_ipc_open(const void *handle, uint64_t *base);
int pg_ipc_close(uint64_t base);

/* Stream-ordered helpers on device memory. */
int pg_memset_async(uint64_t dptr, size_t bytes, uint64_t stream);
int pg_memcpy_htod_async(uint64_t dst, const void *src, size_t bytes, uint64_t stream);
int pg_memcpy_dtoh_async(void *dst, uint64_t src, size_t bytes, uint64_t stream);
int pg_stream_synchronize(uint64_t stream);

/* One launch on host buffers: for each argument i with flags[i] & PG_ARG_IN copy host[i]
 * (bytes[i]) into dev[i]; zero each PG_ARG_ZERO argument; launch; copy each PG_ARG_OUT
 * argument back into host[i]; wait for the stream; then take the module's status word
 * (PG_ERR_KERNEL_STATUS when set). Host buffers should be page-locked for overlap. */
int pg_run_host(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                uint64_t stream, int nargs, const uint64_t *dev, void *const *host,
                const size_t *bytes, const uint32_t *flags);

/* out[0] = the f32 sum of x[0, n), by the grid-kernel plan: `blocks` blocks of
 * PG_GRID_SUM_BLOCK threads each add a grid-stride share into one partial per block, then one
 * block adds the partials. Asynchronous on `stream`; x and out are device pointers (4-byte
 * aligned), n may be 0.
 *
 * No counterpart in the reference. It is for callers that cannot allocate device memory: a
 * plug-in loaded into an application that owns the device's allocator and grants it none; a
 * process whose device memory is all reserved up front by another allocator; a latency-critical
 * path that must not wait on an allocation. ptxgen's own two-kernel sum needs a caller-allocated
 * buffer for its per-block partials. This entry point keeps them in a fixed device array inside
 * the library instead (PG_GRID_SUM_MAX_BLOCKS floats, 16 KiB, held on every GPU where the
 * library's module is loaded until the process exits) and allocates nothing. It does make CUDA
 * calls itself (it launches two kernels), so it must not be called from a host function
 * enqueued on a stream (cudaLaunchHostFunc), where CUDA forbids CUDA calls. blocks must be
 * 1..PG_GRID_SUM_MAX_BLOCKS, else PG_ERR_ARGUMENT. Every call looks up the array's device
 * address in the current context; the first call on a device may load the module, so make it
 * before any stream capture. All calls share the array, so calls that overlap on the GPU (other streams, other
 * threads) race and must not be made. Runtime failures return PG_ERR_RUNTIME. */
#define PG_GRID_SUM_BLOCK 256
#define PG_GRID_SUM_MAX_BLOCKS 4096
int pg_grid_sum_f32_noalloc(uint64_t x, uint64_t n, uint64_t out, uint32_t blocks,
                            uint64_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PTXGEN_B200_H */
