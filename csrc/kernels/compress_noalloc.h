// Allocation-free variant of the delta-compression pipeline.
//
// This entry point has no counterpart in the reference (frane/distrain); it exists for callers of
// this library that cannot allocate device memory: hosts whose device memory is owned by their own
// allocator or reserved in full up front, and loops that must not allocate once they are running
// (a cudaMalloc there can fail, fragment a managed pool, or synchronise the device). Such a caller
// passes only its inputs and outputs; the pipeline's scratch memory is a fixed array inside this
// library.
//
// Contract:
//  * Scratch: DT_COMPRESS_NOALLOC_SCRATCH_BYTES (32 MiB) in a file-scope __device__ array. Every GPU
//    that loads the library holds it until the process exits. The workspace a problem needs is
//    dt_compress_workspace_bytes(nseg, nchunks); larger problems are rejected with -20 (nothing runs).
//  * Set-up: the first call on a device resolves the array's device address (cudaGetSymbolAddress)
//    with that device current and caches it; make that first call before any stream capture.
//  * Sharing: all calls on a device share the one array and it keeps the last call's contents (each
//    call clears it before use). Calls whose GPU work overlaps - concurrent streams, or several host
//    threads - race on it; serialise them (one stream, one caller at a time).
//  * The cached address belongs to the CUDA context that was current at the first call; it does not
//    survive cudaDeviceReset (or any teardown and re-creation of the primary context) - a process that
//    resets a device must not call this entry point on that device again.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
//  * Arguments and outputs are those of dt_compress_begin + dt_compress_finish (one stream), plus
//    n_elems (the element count of master / snap / ef, i.e. the largest cend) and optional per-segment
//    statistics (dt_compress_export_stats layout: nseg * 6 + 4 doubles) in stats_out.
//  * Size limits: n_elems below 2^31 (kept indices are written as plain 32-bit flat offsets; larger
//    buffers need the windowed payload of dt_compress_finish). out_idx / out_val (and out_q) must hold
//    `capacity` entries and out_scales ceil(capacity / quant_block) scales, with
//    capacity >= dt_compress_noalloc_min_capacity(n_elems, nseg, k_fraction) = min(n_elems,
//    ceil(n_elems * k_fraction) + nseg), the most the per-tensor budgets can keep. Should a budget still
//    exceed `capacity` (single-precision rounding of a non-adaptive budget), the surplus entries are not
//    written, stay in error feedback, and dt_error_word is set to 5 (out of bounds).
//  * Returns 0, a CUDA error code, or -10 (invalid argument: nseg, nchunks or n_elems <= 0, k_fraction
//    outside (0, 1]), -20 (workspace exceeds the scratch), -21 (device ordinal >= 64), -22 (n_elems >=
//    2^31), -23 (capacity below the minimum), -24 (quant_block > 0 and not a multiple of 32 up to 512).
//    Nothing runs when an error code is returned.
#pragma once
#include <cuda_runtime.h>

#define DT_COMPRESS_NOALLOC_SCRATCH_BYTES (32ll << 20)

#ifdef __cplusplus
extern "C" {
#endif
long long dt_compress_noalloc_scratch_bytes(void);
long long dt_compress_noalloc_min_capacity(long long n_elems, int nseg, float k_fraction);
int dt_compress_noalloc(const float* master, float* snap, float* ef, const int* cseg, const long long* cstart,
                        const long long* cend, int nchunks, int nseg, const long long* seg_len, long long n_elems,
                        float k_fraction, int adaptive, int* out_idx, float* out_val, signed char* out_q,
                        float* out_scales, int quant_block, long long capacity, double* stats_out,
                        cudaStream_t stream);
#ifdef __cplusplus
}
#endif
