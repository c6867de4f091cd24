// Library-wide device error word: kernels record the first failure (timeout, bounds) here and
// return; the host polls it with dt_get_error() / clears it with dt_clear_error().
#include "common.cuh"

__device__ int dt_error_word = 0;
__device__ int dt_error_site = 0;

DT_API int dt_get_error(int* code, int* site, cudaStream_t stream) {
  DT_CUDA_RET(cudaMemcpyFromSymbolAsync(code, dt_error_word, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
  DT_CUDA_RET(cudaMemcpyFromSymbolAsync(site, dt_error_site, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
  return (int)cudaStreamSynchronize(stream);
}

DT_API int dt_clear_error(cudaStream_t stream) {
  int z = 0;
  DT_CUDA_RET(cudaMemcpyToSymbolAsync(dt_error_word, &z, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
  DT_CUDA_RET(cudaMemcpyToSymbolAsync(dt_error_site, &z, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
  return (int)cudaStreamSynchronize(stream);
}

DT_API int dt_last_cuda_error() { return (int)cudaGetLastError(); }

DT_API const char* dt_cuda_error_string(int e) { return cudaGetErrorString((cudaError_t)e); }

DT_API int dt_device_sm_count(int device) {
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
  return v;
}

DT_API int dt_library_version() { return 1; }

// Installed driver and linked runtime versions (e.g. 12080 = 12.8); 0 when no driver is present.
DT_API int dt_cuda_versions(int* driver, int* runtime) {
  *driver = 0;
  *runtime = 0;
  cudaDriverGetVersion(driver);
  cudaRuntimeGetVersion(runtime);
  return 0;
}
