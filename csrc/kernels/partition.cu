// SM partitions for the coordinator's merge: a green context that owns a disjoint group of SMs, and a
// stream in it. Kernels launched into that stream run only on the group's SMs, so a merge never takes
// more than that share of the GPU from the training kernels of the node it shares the device with.
//
// The partition is made with the driver's resource API (device SM resource -> split by count ->
// descriptor -> green context -> stream), resolved through cudaGetDriverEntryPoint so the library does
// not link libcuda. The group size is rounded up by the driver (multiples of 8 SMs on this
// architecture); the granted count is returned.
//
// dt_smid_probe records the SM that ran each block, which the tests use to check that a stream's
// kernels stay inside its partition.
#include <cuda.h>
#include <mutex>
#include "common.cuh"

namespace {

typedef CUresult (*PFN_devGet)(CUdevice*, int);
typedef CUresult (*PFN_devRes)(CUdevice, CUdevResource*, CUdevResourceType);
typedef CUresult (*PFN_split)(CUdevResource*, unsigned int*, const CUdevResource*, CUdevResource*, unsigned int,
                              unsigned int);
typedef CUresult (*PFN_desc)(CUdevResourceDesc*, CUdevResource*, unsigned int);
typedef CUresult (*PFN_gcreate)(CUgreenCtx*, CUdevResourceDesc, CUdevice, unsigned int);
typedef CUresult (*PFN_gstream)(CUstream*, CUgreenCtx, unsigned int, int);
typedef CUresult (*PFN_gdestroy)(CUgreenCtx);
typedef CUresult (*PFN_sdestroy)(CUstream);

struct Drv {
  PFN_devGet dev_get = nullptr;
  PFN_devRes dev_res = nullptr;
  PFN_split split = nullptr;
  PFN_desc desc = nullptr;
  PFN_gcreate gcreate = nullptr;
  PFN_gstream gstream = nullptr;
  PFN_gdestroy gdestroy = nullptr;
  PFN_sdestroy sdestroy = nullptr;
  bool ok = false;
};
Drv g_drv;
std::once_flag g_drv_once;

template <typename F>
bool entry(const char* name, F& out) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &fn, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return false;
  out = reinterpret_cast<F>(fn);
  return true;
}

const Drv& drv() {
  std::call_once(g_drv_once, [] {
    Drv d;
    d.ok = entry("cuDeviceGet", d.dev_get) && entry("cuDeviceGetDevResource", d.dev_res) &&
           entry("cuDevSmResourceSplitByCount", d.split) && entry("cuDevResourceGenerateDesc", d.desc) &&
           entry("cuGreenCtxCreate", d.gcreate) && entry("cuGreenCtxStreamCreate", d.gstream) &&
           entry("cuGreenCtxDestroy", d.gdestroy) && entry("cuStreamDestroy", d.sdestroy);
    g_drv = d;
  });
  return g_drv;
}

__global__ void smid_probe_kernel(int* __restrict__ out, long long spin_ns) {
  if (threadIdx.x != 0) return;
  unsigned sm;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
  out[blockIdx.x] = (int)sm;
  // stay resident for a while (bounded by the timer) so that later blocks have to spread over SMs
  const uint64_t t0 = dt_globaltimer();
  while (dt_globaltimer() - t0 < (uint64_t)spin_ns) {}
}

}  // namespace

// Creates a green context on `device` owning at least `sms` SMs and a non-blocking stream of the given
// priority in it. Returns 0 and the stream, an opaque handle and the granted SM count (and the device's
// total); -1 when the driver lacks the API, -2 on bad arguments, a CUresult (>0) from the failing call.
DT_API int dt_sm_partition_create(int device, int sms, int priority, void** stream, void** handle, int* granted,
                                  int* total) {
  const Drv& d = drv();
  if (!d.ok) return -1;
  if (sms <= 0 || !stream || !handle || !granted || !total) return -2;
  DT_CUDA_RET(cudaFree(nullptr));  // the primary context exists before the green context retains it
  CUdevice dev;
  CUresult r = d.dev_get(&dev, device);
  if (r != CUDA_SUCCESS) return (int)r;
  CUdevResource all;
  if ((r = d.dev_res(dev, &all, CU_DEV_RESOURCE_TYPE_SM)) != CUDA_SUCCESS) return (int)r;
  if ((unsigned)sms >= all.sm.smCount) return -2;
  CUdevResource part, rest;
  unsigned int n = 1;
  if ((r = d.split(&part, &n, &all, &rest, 0, (unsigned)sms)) != CUDA_SUCCESS) return (int)r;
  if (n < 1) return -2;
  CUdevResourceDesc desc;
  if ((r = d.desc(&desc, &part, 1)) != CUDA_SUCCESS) return (int)r;
  CUgreenCtx g;
  if ((r = d.gcreate(&g, desc, dev, CU_GREEN_CTX_DEFAULT_STREAM)) != CUDA_SUCCESS) return (int)r;
  CUstream s;
  if ((r = d.gstream(&s, g, CU_STREAM_NON_BLOCKING, priority)) != CUDA_SUCCESS) {
    d.gdestroy(g);
    return (int)r;
  }
  *stream = (void*)s;
  *handle = (void*)g;
  *granted = (int)part.sm.smCount;
  *total = (int)all.sm.smCount;
  return 0;
}

// Destroys the stream and the green context (the caller has synchronised the stream).
DT_API int dt_sm_partition_destroy(void* handle, void* stream) {
  const Drv& d = drv();
  if (!d.ok) return -1;
  if (stream) d.sdestroy((CUstream)stream);
  if (handle) d.gdestroy((CUgreenCtx)handle);
  return 0;
}

// Writes the SM id of each of `nblocks` blocks to out[block]; each block stays resident ~spin_ns.
DT_API int dt_smid_probe(int* out, int nblocks, long long spin_ns, cudaStream_t stream) {
  if (!out || nblocks <= 0 || spin_ns < 0 || spin_ns > 100000000LL) return -10;
  smid_probe_kernel<<<nblocks, 32, 0, stream>>>(out, spin_ns);
  return (int)cudaGetLastError();
}

// Records `site` as a DT_ERR_BAD_ARG in the library's error word from a kernel on `stream` (tests use it to
// check which error word a partition's kernels write).
__global__ void raise_error_kernel(int site) { dt_set_error(DT_ERR_BAD_ARG, site); }
DT_API int dt_raise_error(int site, cudaStream_t stream) {
  raise_error_kernel<<<1, 1, 0, stream>>>(site);
  return (int)cudaGetLastError();
}
