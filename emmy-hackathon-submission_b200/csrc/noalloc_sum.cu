// pg_grid_sum_f32_noalloc: the grid-kernel sum (per-block partials, then one block over them)
// for callers that cannot allocate device memory.
//
// The two-kernel sum ptxgen emits for the grid-kernel reduce plan keeps its per-block partials
// in an intermediate buffer that the caller allocates. Some callers cannot do that: a plug-in
// loaded into an application whose allocator owns the whole device and grants it nothing, a
// process whose device memory is reserved up front, and code that must not pay an allocation's
// synchronisation on a latency-critical path. This entry point runs the same plan with the
// partials in one file-scope device array instead, so the caller passes only the input and the
// output. It still launches kernels, so it is no use inside a stream's host function, where CUDA
// forbids every CUDA call.
//
// The array holds PG_GRID_SUM_MAX_BLOCKS floats (16 KiB). It belongs to this library's device
// module: every GPU on which the module is loaded holds it until the process exits. Every call
// on a device shares it, and it keeps the last call's contents; a call writes every slot it then
// reads (slot b by block b of the first kernel), so nothing needs clearing between calls. Calls
// whose kernels overlap on the GPU (two streams, or two host threads on one device) race on the
// array and must not be made.
//
// Host code cannot use the array's name as a device address (there it names a host-side stand-in
// for the symbol). Every call asks the runtime for the array's device address in the current
// context (cudaGetSymbolAddress); the first call on a device may load this library's module, so
// it should come before any stream capture. Nothing is kept between calls, so a call after
// cudaDeviceReset finds the array where the module was loaded again.
//
// The summation order is the emitted kernels': each thread adds its grid-stride share in index
// order, a warp combines its lanes by the xor butterfly of strides 16..1 (v = v + other), the
// block's warps are combined by the halving tree over the per-warp slots, and the final block
// does the same over the partials.

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "../../include/ptxgen_b200.h"

// Records `msg` as the calling thread's last error (launcher.cpp) and returns `code`.
int pg_detail_fail(int code, const char *msg);

namespace {

constexpr int kBlock = PG_GRID_SUM_BLOCK;
constexpr int kWarps = kBlock / 32;
// block_sum's second stage is an xor butterfly over one warp's lanes from kWarps / 2 down: it
// needs whole warps, at most 32 of them, a power of two
static_assert(kBlock % 32 == 0 && kWarps >= 1 && kWarps <= 32 && (kWarps & (kWarps - 1)) == 0,
              "PG_GRID_SUM_BLOCK must be 32 times a power of two, at most 1024");

static __device__ __align__(256) float g_partials[PG_GRID_SUM_MAX_BLOCKS];

__device__ __forceinline__ float block_sum(float v, float *slots) {
  const unsigned lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off; off >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, off);
  if (lane == 0) slots[warp] = v;
  __syncthreads();
  float w = 0.0f;
  if (warp == 0) {
    w = lane < kWarps ? slots[lane] : 0.0f;
#pragma unroll
    for (int off = kWarps / 2; off; off >>= 1) w = w + __shfl_xor_sync(0xffffffffu, w, off);
  }
  return w;  // the block's total in thread 0
}

// Block b sums x[b*kBlock + t + k*kBlock*gridDim.x] over its threads t and stores the total in
// partials[b].
__global__ void __launch_bounds__(kBlock) grid_sum_partials(const float *__restrict__ x,
                                                            uint64_t n,
                                                            float *__restrict__ partials) {
  __shared__ float slots[kWarps];
  const uint64_t stride = static_cast<uint64_t>(kBlock) * gridDim.x;
  float acc = 0.0f;
  for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kBlock + threadIdx.x; i < n; i += stride)
    acc = acc + __ldg(x + i);
  const float total = block_sum(acc, slots);
  if (threadIdx.x == 0) partials[blockIdx.x] = total;
}

// One block sums partials[0, blocks) into out[0].
__global__ void __launch_bounds__(kBlock) grid_sum_final(const float *__restrict__ partials,
                                                         uint32_t blocks,
                                                         float *__restrict__ out) {
  __shared__ float slots[kWarps];
  float acc = 0.0f;
  for (uint32_t i = threadIdx.x; i < blocks; i += kBlock) acc = acc + partials[i];
  const float total = block_sum(acc, slots);
  if (threadIdx.x == 0) out[0] = total;
}

int runtime_fail(cudaError_t e, const char *what) {
  char buf[512];
  snprintf(buf, sizeof buf, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  return pg_detail_fail(PG_ERR_RUNTIME, buf);
}

// The device address of g_partials in the current context, looked up on every call (a host-side
// table lookup that allocates nothing), so a call after the context was reset and the module
// loaded again gets the new address.
int scratch_address(float **out) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_partials);
  if (e != cudaSuccess) return runtime_fail(e, "cudaGetSymbolAddress(g_partials)");
  *out = static_cast<float *>(p);
  return PG_OK;
}

}  // namespace

extern "C" int pg_grid_sum_f32_noalloc(uint64_t x, uint64_t n, uint64_t out, uint32_t blocks,
                                       uint64_t stream) {
  char buf[256];
  if (blocks == 0 || blocks > PG_GRID_SUM_MAX_BLOCKS) {
    snprintf(buf, sizeof buf,
             "pg_grid_sum_f32_noalloc: blocks = %u, want 1..%d (the partials array's size)",
             blocks, PG_GRID_SUM_MAX_BLOCKS);
    return pg_detail_fail(PG_ERR_ARGUMENT, buf);
  }
  if (!out || (n && !x))
    return pg_detail_fail(PG_ERR_ARGUMENT, "pg_grid_sum_f32_noalloc: null pointer");
  if ((x | out) & 3u)
    return pg_detail_fail(PG_ERR_ARGUMENT,
                          "pg_grid_sum_f32_noalloc: x and out must be 4-byte aligned");
  float *partials = nullptr;
  int rc = scratch_address(&partials);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(stream));
  grid_sum_partials<<<blocks, kBlock, 0, s>>>(
      reinterpret_cast<const float *>(static_cast<uintptr_t>(x)), n, partials);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return runtime_fail(e, "grid_sum_partials launch");
  grid_sum_final<<<1, kBlock, 0, s>>>(partials, blocks,
                                      reinterpret_cast<float *>(static_cast<uintptr_t>(out)));
  e = cudaGetLastError();
  if (e != cudaSuccess) return runtime_fail(e, "grid_sum_final launch");
  return PG_OK;
}
