// The C-ABI launcher for ptxgen-emitted PTX (see include/ptxgen_b200.h).
//
// libcuda is opened with dlopen at pg_init, not linked, so this library loads (and its symbols
// can be inspected) on a machine without a GPU driver. Only driver-API calls are used: the
// primary context of the device is shared with the CUDA runtime PyTorch runs on, so device
// pointers and streams from PyTorch are valid here. Nothing here allocates device memory.

#include <cuda.h>
#include <dlfcn.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/ptxgen_b200.h"

namespace {

thread_local std::string g_error = "no error";

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

struct Driver {
  bool loaded = false;
  void *lib = nullptr;
  CUresult (*Init)(unsigned);
  CUresult (*DeviceGet)(CUdevice *, int);
  CUresult (*PrimaryCtxRetain)(CUcontext *, CUdevice);
  CUresult (*CtxSetCurrent)(CUcontext);
  CUresult (*CtxGetCurrent)(CUcontext *);
  CUresult (*ModuleLoadDataEx)(CUmodule *, const void *, unsigned, CUjit_option *, void **);
  CUresult (*ModuleUnload)(CUmodule);
  CUresult (*ModuleGetFunction)(CUfunction *, CUmodule, const char *);
  CUresult (*ModuleGetGlobal)(CUdeviceptr *, size_t *, CUmodule, const char *);
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int);
  CUresult (*LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned,
                           unsigned, unsigned, CUstream, void **, void **);
  CUresult (*MemsetD8Async)(CUdeviceptr, unsigned char, size_t, CUstream);
  CUresult (*MemcpyHtoDAsync)(CUdeviceptr, const void *, size_t, CUstream);
  CUresult (*MemcpyDtoHAsync)(void *, CUdeviceptr, size_t, CUstream);
  CUresult (*MemcpyHtoD)(CUdeviceptr, const void *, size_t);
  CUresult (*MemcpyDtoH)(void *, CUdeviceptr, size_t);
  CUresult (*StreamSynchronize)(CUstream);
  CUresult (*CtxSynchronize)(void);
  CUresult (*TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
  CUresult (*OccupancyMaxActiveClusters)(int *, CUfunction, const CUlaunchConfig *);
  CUresult (*LaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **, void **);
  CUresult (*EventCreate)(CUevent *, unsigned);
  CUresult (*EventRecord)(CUevent, CUstream);
  CUresult (*EventSynchronize)(CUevent);
  CUresult (*EventElapsedTime)(float *, CUevent, CUevent);
  CUresult (*EventDestroy)(CUevent);
  CUresult (*MemGetAddressRange)(CUdeviceptr *, size_t *, CUdeviceptr);
  CUresult (*IpcGetMemHandle)(CUipcMemHandle *, CUdeviceptr);
  CUresult (*IpcOpenMemHandle)(CUdeviceptr *, CUipcMemHandle, unsigned);
  CUresult (*IpcCloseMemHandle)(CUdeviceptr);
  CUresult (*GetErrorName)(CUresult, const char **);
  CUresult (*GetErrorString)(CUresult, const char **);
};

Driver g_drv;
std::mutex g_mu;
CUcontext g_ctx = nullptr;

template <class F>
bool sym(F &fn, const char *name) {
  fn = reinterpret_cast<F>(dlsym(g_drv.lib, name));
  return fn != nullptr;
}

int load_driver() {
  if (g_drv.loaded) return PG_OK;
  g_drv.lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_LOCAL);
  if (!g_drv.lib) return fail(PG_ERR_NO_DRIVER, "dlopen(libcuda.so.1): %s", dlerror());
  const char *missing = nullptr;
#define PG_SYM(field, name) \
  if (!missing && !sym(g_drv.field, name)) missing = name;
  PG_SYM(Init, "cuInit")
  PG_SYM(DeviceGet, "cuDeviceGet")
  PG_SYM(PrimaryCtxRetain, "cuDevicePrimaryCtxRetain")
  PG_SYM(CtxSetCurrent, "cuCtxSetCurrent")
  PG_SYM(CtxGetCurrent, "cuCtxGetCurrent")
  PG_SYM(ModuleLoadDataEx, "cuModuleLoadDataEx")
  PG_SYM(ModuleUnload, "cuModuleUnload")
  PG_SYM(ModuleGetFunction, "cuModuleGetFunction")
  PG_SYM(ModuleGetGlobal, "cuModuleGetGlobal_v2")
  PG_SYM(FuncSetAttribute, "cuFuncSetAttribute")
  PG_SYM(LaunchKernel, "cuLaunchKernel")
  PG_SYM(MemsetD8Async, "cuMemsetD8Async")
  PG_SYM(MemcpyHtoDAsync, "cuMemcpyHtoDAsync_v2")
  PG_SYM(MemcpyDtoHAsync, "cuMemcpyDtoHAsync_v2")
  PG_SYM(MemcpyHtoD, "cuMemcpyHtoD_v2")
  PG_SYM(MemcpyDtoH, "cuMemcpyDtoH_v2")
  PG_SYM(StreamSynchronize, "cuStreamSynchronize")
  PG_SYM(CtxSynchronize, "cuCtxSynchronize")
  PG_SYM(TensorMapEncodeTiled, "cuTensorMapEncodeTiled")
  PG_SYM(OccupancyMaxActiveClusters, "cuOccupancyMaxActiveClusters")
  PG_SYM(LaunchKernelEx, "cuLaunchKernelEx")
  PG_SYM(EventCreate, "cuEventCreate")
  PG_SYM(EventRecord, "cuEventRecord")
  PG_SYM(EventSynchronize, "cuEventSynchronize")
  PG_SYM(EventElapsedTime, "cuEventElapsedTime")
  PG_SYM(EventDestroy, "cuEventDestroy_v2")
  PG_SYM(MemGetAddressRange, "cuMemGetAddressRange_v2")
  PG_SYM(IpcGetMemHandle, "cuIpcGetMemHandle")
  PG_SYM(IpcOpenMemHandle, "cuIpcOpenMemHandle_v2")
  PG_SYM(IpcCloseMemHandle, "cuIpcCloseMemHandle")
  PG_SYM(GetErrorName, "cuGetErrorName")
  PG_SYM(GetErrorString, "cuGetErrorString")
#undef PG_SYM
  if (missing) return fail(PG_ERR_NO_DRIVER, "libcuda.so.1 has no %s", missing);
  g_drv.loaded = true;
  return PG_OK;
}

int cu_fail(CUresult r, const char *what) {
  const char *name = "CUDA_ERROR_UNKNOWN", *text = "";
  if (g_drv.GetErrorName) g_drv.GetErrorName(r, &name);
  if (g_drv.GetErrorString) g_drv.GetErrorString(r, &text);
  return fail(static_cast<int>(r), "%s: %s (%s)", what, name, text);
}

#define PG_CU(call, what)                          \
  do {                                             \
    CUresult r_ = (call);                          \
    if (r_ != CUDA_SUCCESS) return cu_fail(r_, what); \
  } while (0)

int ensure_current() {
  if (!g_drv.loaded || !g_ctx) return fail(PG_ERR_NOT_INITIALISED, "pg_init has not run");
  CUcontext cur = nullptr;
  g_drv.CtxGetCurrent(&cur);
  if (cur != g_ctx) PG_CU(g_drv.CtxSetCurrent(g_ctx), "cuCtxSetCurrent");
  return PG_OK;
}

struct TmapKey {
  int dtype, rank, swizzle;
  uint64_t base, dims[5], strides[4];
  uint32_t box[5];
  bool operator==(const TmapKey &o) const { return std::memcmp(this, &o, sizeof o) == 0; }
};

}  // namespace

// Records `msg` as this thread's last error and returns `code`: the error channel of the entry
// points defined in other translation units (noalloc_sum.cu). Not exported.
__attribute__((visibility("hidden"))) int pg_detail_fail(int code, const char *msg) {
  return fail(code, "%s", msg);
}

struct pg_module {
  CUmodule mod = nullptr;
  std::unordered_map<std::string, TmapKey> filled;
  CUdeviceptr status = 0;
  bool status_known = false;
};

struct pg_kernel {
  CUfunction fn = nullptr;
  pg_module *module = nullptr;
  int smem_optin = 48 * 1024;
};

extern "C" {

const char *pg_last_error(void) { return g_error.c_str(); }

int pg_init(int device) {
  std::lock_guard<std::mutex> lock(g_mu);
  int rc = load_driver();
  if (rc) return rc;
  PG_CU(g_drv.Init(0), "cuInit");
  CUdevice dev;
  PG_CU(g_drv.DeviceGet(&dev, device), "cuDeviceGet");
  CUcontext ctx;
  PG_CU(g_drv.PrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
  PG_CU(g_drv.CtxSetCurrent(ctx), "cuCtxSetCurrent");
  g_ctx = ctx;
  return PG_OK;
}

int pg_module_load(const char *ptx, pg_module **out) {
  if (!ptx || !out) return fail(PG_ERR_ARGUMENT, "pg_module_load: null argument");
  int rc = ensure_current();
  if (rc) return rc;
  static thread_local char log[1 << 16];
  log[0] = 0;
  CUjit_option opts[] = {CU_JIT_ERROR_LOG_BUFFER, CU_JIT_ERROR_LOG_BUFFER_SIZE_BYTES};
  void *vals[] = {log, reinterpret_cast<void *>(static_cast<uintptr_t>(sizeof log))};
  CUmodule mod = nullptr;
  CUresult r = g_drv.ModuleLoadDataEx(&mod, ptx, 2, opts, vals);
  if (r != CUDA_SUCCESS) {
    cu_fail(r, "cuModuleLoadDataEx");
    g_error += "\nJIT log:\n";
    g_error += log;
    return static_cast<int>(r);
  }
  auto *m = new pg_module;
  m->mod = mod;
  *out = m;
  return PG_OK;
}

int pg_module_unload(pg_module *module) {
  if (!module) return fail(PG_ERR_ARGUMENT, "pg_module_unload: null module");
  int rc = ensure_current();
  if (rc) return rc;
  CUresult r = g_drv.ModuleUnload(module->mod);
  delete module;
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuModuleUnload");
  return PG_OK;
}

int pg_kernel_get(pg_module *module, const char *entry, pg_kernel **out) {
  if (!module || !entry || !out) return fail(PG_ERR_ARGUMENT, "pg_kernel_get: null argument");
  int rc = ensure_current();
  if (rc) return rc;
  CUfunction fn;
  CUresult r = g_drv.ModuleGetFunction(&fn, module->mod, entry);
  if (r == CUDA_ERROR_NOT_FOUND) return fail(PG_ERR_NOT_FOUND, "no entry %s in module", entry);
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuModuleGetFunction");
  auto *k = new pg_kernel;
  k->fn = fn;
  k->module = module;
  *out = k;
  return PG_OK;
}

int pg_kernel_launch(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                     uint64_t stream, const uint64_t *ptrs, int nptrs) {
  return pg_kernel_launch_ex(kernel, grid, block, smem_bytes, stream, ptrs, nptrs, 0);
}

int pg_kernel_launch_ex(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                        uint64_t stream, const uint64_t *ptrs, int nptrs, uint32_t flags) {
  if (!kernel || (nptrs > 0 && !ptrs) || nptrs < 0 || nptrs > 256)
    return fail(PG_ERR_ARGUMENT, "pg_kernel_launch: bad kernel or arguments");
  if (grid == 0 || block == 0 || block > 1024)
    return fail(PG_ERR_ARGUMENT, "pg_kernel_launch: grid %u block %u", grid, block);
  if (flags & ~static_cast<uint32_t>(PG_LAUNCH_EARLY))
    return fail(PG_ERR_ARGUMENT, "pg_kernel_launch_ex: unknown flags 0x%x", flags);
  int rc = ensure_current();
  if (rc) return rc;
  if (static_cast<int>(smem_bytes) > kernel->smem_optin) {
    PG_CU(g_drv.FuncSetAttribute(kernel->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                 static_cast<int>(smem_bytes)),
          "cuFuncSetAttribute(MAX_DYNAMIC_SHARED_SIZE_BYTES)");
    kernel->smem_optin = static_cast<int>(smem_bytes);
  }
  std::vector<uint64_t> vals(ptrs, ptrs + nptrs);
  std::vector<void *> args(nptrs);
  for (int i = 0; i < nptrs; ++i) args[i] = &vals[i];
  if (!(flags & PG_LAUNCH_EARLY)) {
    PG_CU(g_drv.LaunchKernel(kernel->fn, grid, 1, 1, block, 1, 1, smem_bytes,
                             reinterpret_cast<CUstream>(stream), args.data(), nullptr),
          "cuLaunchKernel");
    return PG_OK;
  }
  // programmatic stream serialization: the kernel may start once the previous kernel on the
  // stream has triggered (griddepcontrol.launch_dependents) or ended
  CUlaunchAttribute attr;
  std::memset(&attr, 0, sizeof attr);
  attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
  attr.value.programmaticStreamSerializationAllowed = 1;
  CUlaunchConfig cfg;
  std::memset(&cfg, 0, sizeof cfg);
  cfg.gridDimX = grid;
  cfg.gridDimY = cfg.gridDimZ = 1;
  cfg.blockDimX = block;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = smem_bytes;
  cfg.hStream = reinterpret_cast<CUstream>(stream);
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  PG_CU(g_drv.LaunchKernelEx(&cfg, kernel->fn, args.data(), nullptr), "cuLaunchKernelEx");
  return PG_OK;
}

int pg_kernel_max_clusters(pg_kernel *kernel, uint32_t block, uint32_t smem_bytes,
                           uint32_t cluster, int *out) {
  if (!kernel || !out || block == 0 || block > 1024 || cluster == 0 || cluster > 16)
    return fail(PG_ERR_ARGUMENT, "pg_kernel_max_clusters: bad arguments");
  int rc = ensure_current();
  if (rc) return rc;
  if (static_cast<int>(smem_bytes) > kernel->smem_optin) {
    PG_CU(g_drv.FuncSetAttribute(kernel->fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                 static_cast<int>(smem_bytes)),
          "cuFuncSetAttribute(MAX_DYNAMIC_SHARED_SIZE_BYTES)");
    kernel->smem_optin = static_cast<int>(smem_bytes);
  }
  CUlaunchAttribute attr;
  std::memset(&attr, 0, sizeof attr);
  attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
  attr.value.clusterDim.x = cluster;
  attr.value.clusterDim.y = 1;
  attr.value.clusterDim.z = 1;
  CUlaunchConfig cfg;
  std::memset(&cfg, 0, sizeof cfg);
  cfg.gridDimX = cluster;
  cfg.gridDimY = cfg.gridDimZ = 1;
  cfg.blockDimX = block;
  cfg.blockDimY = cfg.blockDimZ = 1;
  cfg.sharedMemBytes = smem_bytes;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  PG_CU(g_drv.OccupancyMaxActiveClusters(out, kernel->fn, &cfg),
        "cuOccupancyMaxActiveClusters");
  return PG_OK;
}

int pg_kernel_time(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                   uint64_t stream, const uint64_t *ptrs, int nptrs, int warmup, int reps,
                   float *ms_out) {
  if (!kernel || warmup < 0 || reps < 1 || reps > 100000 || !ms_out)
    return fail(PG_ERR_ARGUMENT, "pg_kernel_time: bad arguments");
  int rc;
  for (int i = 0; i < warmup; ++i)
    if ((rc = pg_kernel_launch(kernel, grid, block, smem_bytes, stream, ptrs, nptrs))) return rc;
  std::vector<CUevent> ev(2 * static_cast<size_t>(reps), nullptr);
  CUstream s = reinterpret_cast<CUstream>(stream);
  auto destroy = [&ev]() {
    for (CUevent e : ev)
      if (e) g_drv.EventDestroy(e);
  };
  CUresult r = CUDA_SUCCESS;
  for (size_t i = 0; i < ev.size() && r == CUDA_SUCCESS; ++i) r = g_drv.EventCreate(&ev[i], 0);
  if (r != CUDA_SUCCESS) {
    destroy();
    return cu_fail(r, "cuEventCreate");
  }
  for (int i = 0; i < reps; ++i) {
    if ((r = g_drv.EventRecord(ev[2 * i], s)) != CUDA_SUCCESS) break;
    if ((rc = pg_kernel_launch(kernel, grid, block, smem_bytes, stream, ptrs, nptrs))) {
      destroy();
      return rc;
    }
    if ((r = g_drv.EventRecord(ev[2 * i + 1], s)) != CUDA_SUCCESS) break;
  }
  if (r == CUDA_SUCCESS) r = g_drv.EventSynchronize(ev.back());
  for (int i = 0; i < reps && r == CUDA_SUCCESS; ++i)
    r = g_drv.EventElapsedTime(&ms_out[i], ev[2 * i], ev[2 * i + 1]);
  destroy();
  if (r != CUDA_SUCCESS) return cu_fail(r, "timing events");
  return PG_OK;
}

int pg_tensormap_fill(pg_module *module, const char *symbol, int dtype, int rank, uint64_t base,
                      const uint64_t *dims, const uint64_t *strides_bytes, const uint32_t *box,
                      int swizzle_bytes) {
  if (!module || !symbol || !dims || !box || rank < 1 || rank > 5 ||
      (rank > 1 && !strides_bytes))
    return fail(PG_ERR_ARGUMENT, "pg_tensormap_fill: bad arguments");
  int rc = ensure_current();
  if (rc) return rc;
  CUtensorMapDataType dt;
  switch (dtype) {
    case PG_DT_U8: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case PG_DT_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case PG_DT_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case PG_DT_F32: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: return fail(PG_ERR_ARGUMENT, "pg_tensormap_fill: dtype %d", dtype);
  }
  CUtensorMapSwizzle sw;
  switch (swizzle_bytes) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return fail(PG_ERR_ARGUMENT, "pg_tensormap_fill: swizzle %d", swizzle_bytes);
  }
  TmapKey key{};
  key.dtype = dtype;
  key.rank = rank;
  key.swizzle = swizzle_bytes;
  key.base = base;
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.strides[i] = strides_bytes[i];
  }
  auto it = module->filled.find(symbol);
  if (it != module->filled.end() && it->second == key) return PG_OK;

  CUdeviceptr dst;
  size_t bytes;
  CUresult r = g_drv.ModuleGetGlobal(&dst, &bytes, module->mod, symbol);
  if (r == CUDA_ERROR_NOT_FOUND) return fail(PG_ERR_NOT_FOUND, "no .global %s in module", symbol);
  if (r != CUDA_SUCCESS) return cu_fail(r, "cuModuleGetGlobal");
  if (bytes < sizeof(CUtensorMap))
    return fail(PG_ERR_ARGUMENT, ".global %s holds %zu bytes, a tensor map needs %zu", symbol,
                bytes, sizeof(CUtensorMap));
  CUtensorMap map;
  cuuint32_t estride[5] = {1, 1, 1, 1, 1};
  PG_CU(g_drv.TensorMapEncodeTiled(&map, dt, static_cast<cuuint32_t>(rank),
                                   reinterpret_cast<void *>(base), dims, strides_bytes, box,
                                   estride, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE),
        "cuTensorMapEncodeTiled");
  // Synchronous copy: kernels launched earlier that read the old map have finished reading
  // it by the time the copy lands, since it waits for the device to go idle.
  PG_CU(g_drv.CtxSynchronize(), "cuCtxSynchronize");
  PG_CU(g_drv.MemcpyHtoD(dst, &map, sizeof map), "cuMemcpyHtoD(tensor map)");
  module->filled[symbol] = key;
  return PG_OK;
}

int pg_global_write(pg_module *module, const char *symbol, const void *data, size_t bytes) {
  if (!module || !symbol || (bytes && !data))
    return fail(PG_ERR_ARGUMENT, "pg_global_write: null argument");
  int rc = ensure_current();
  if (rc) return rc;
  CUdeviceptr dst = 0;
  size_t size = 0;
  CUresult r = g_drv.ModuleGetGlobal(&dst, &size, module->mod, symbol);
  if (r != CUDA_SUCCESS) return fail(PG_ERR_NOT_FOUND, "pg_global_write: no .global %s", symbol);
  if (bytes > size)
    return fail(PG_ERR_ARGUMENT, "pg_global_write: %zu bytes into %s of %zu", bytes, symbol, size);
  if (bytes) PG_CU(g_drv.MemcpyHtoD(dst, data, bytes), "cuMemcpyHtoD(global)");
  return PG_OK;
}

int pg_status_take(pg_module *module, uint32_t *status) {
  if (!module || !status) return fail(PG_ERR_ARGUMENT, "pg_status_take: null argument");
  int rc = ensure_current();
  if (rc) return rc;
  *status = 0;
  if (!module->status_known) {
    size_t bytes = 0;
    CUresult r = g_drv.ModuleGetGlobal(&module->status, &bytes, module->mod, "ptxgen_status");
    if (r != CUDA_SUCCESS) module->status = 0;
    module->status_known = true;
  }
  if (!module->status) return PG_OK;
  PG_CU(g_drv.MemcpyDtoH(status, module->status, sizeof *status), "cuMemcpyDtoH(status)");
  if (*status) {
    uint32_t zero = 0;
    PG_CU(g_drv.MemcpyHtoD(module->status, &zero, sizeof zero), "cuMemcpyHtoD(status)");
  }
  return PG_OK;
}

int pg_ipc_handle(uint64_t ptr, void *handle, uint64_t *offset) {
  if (!ptr || !handle || !offset) return fail(PG_ERR_ARGUMENT, "pg_ipc_handle: null argument");
  int rc = ensure_current();
  if (rc) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  PG_CU(g_drv.MemGetAddressRange(&base, &size, ptr), "cuMemGetAddressRange");
  CUipcMemHandle h;
  PG_CU(g_drv.IpcGetMemHandle(&h, base), "cuIpcGetMemHandle");
  std::memcpy(handle, h.reserved, sizeof h.reserved);
  *offset = ptr - base;
  return PG_OK;
}

int pg_ipc_open(const void *handle, uint64_t *base) {
  if (!handle || !base) return fail(PG_ERR_ARGUMENT, "pg_ipc_open: null argument");
  int rc = ensure_current();
  if (rc) return rc;
  CUipcMemHandle h;
  std::memcpy(h.reserved, handle, sizeof h.reserved);
  CUdeviceptr p = 0;
  PG_CU(g_drv.IpcOpenMemHandle(&p, h, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS), "cuIpcOpenMemHandle");
  *base = p;
  return PG_OK;
}

int pg_ipc_close(uint64_t base) {
  if (!base) return fail(PG_ERR_ARGUMENT, "pg_ipc_close: null base");
  int rc = ensure_current();
  if (rc) return rc;
  PG_CU(g_drv.IpcCloseMemHandle(base), "cuIpcCloseMemHandle");
  return PG_OK;
}

int pg_memset_async(uint64_t dptr, size_t bytes, uint64_t stream) {
  int rc = ensure_current();
  if (rc) return rc;
  PG_CU(g_drv.MemsetD8Async(dptr, 0, bytes, reinterpret_cast<CUstream>(stream)),
        "cuMemsetD8Async");
  return PG_OK;
}

int pg_memcpy_htod_async(uint64_t dst, const void *src, size_t bytes, uint64_t stream) {
  int rc = ensure_current();
  if (rc) return rc;
  PG_CU(g_drv.MemcpyHtoDAsync(dst, src, bytes, reinterpret_cast<CUstream>(stream)),
        "cuMemcpyHtoDAsync");
  return PG_OK;
}

int pg_memcpy_dtoh_async(void *dst, uint64_t src, size_t bytes, uint64_t stream) {
  int rc = ensure_current();
  if (rc) return rc;
  PG_CU(g_drv.MemcpyDtoHAsync(dst, src, bytes, reinterpret_cast<CUstream>(stream)),
        "cuMemcpyDtoHAsync");
  return PG_OK;
}

int pg_stream_synchronize(uint64_t stream) {
  int rc = ensure_current();
  if (rc) return rc;
  PG_CU(g_drv.StreamSynchronize(reinterpret_cast<CUstream>(stream)), "cuStreamSynchronize");
  return PG_OK;
}

int pg_run_host(pg_kernel *kernel, uint32_t grid, uint32_t block, uint32_t smem_bytes,
                uint64_t stream, int nargs, const uint64_t *dev, void *const *host,
                const size_t *bytes, const uint32_t *flags) {
  if (!kernel || nargs < 0 || (nargs > 0 && (!dev || !host || !bytes || !flags)))
    return fail(PG_ERR_ARGUMENT, "pg_run_host: bad arguments");
  int rc;
  for (int i = 0; i < nargs; ++i) {
    if ((flags[i] & PG_ARG_IN) && host[i] &&
        (rc = pg_memcpy_htod_async(dev[i], host[i], bytes[i], stream)))
      return rc;
    if ((flags[i] & PG_ARG_ZERO) && (rc = pg_memset_async(dev[i], bytes[i], stream))) return rc;
  }
  if ((rc = pg_kernel_launch(kernel, grid, block, smem_bytes, stream, dev, nargs))) return rc;
  for (int i = 0; i < nargs; ++i)
    if ((flags[i] & PG_ARG_OUT) && host[i] &&
        (rc = pg_memcpy_dtoh_async(host[i], dev[i], bytes[i], stream)))
      return rc;
  if ((rc = pg_stream_synchronize(stream))) return rc;
  uint32_t status = 0;
  if ((rc = pg_status_take(kernel->module, &status))) return rc;
  if (status) return fail(PG_ERR_KERNEL_STATUS, "kernel status word 0x%08x", status);
  return PG_OK;
}

}  // extern "C"
