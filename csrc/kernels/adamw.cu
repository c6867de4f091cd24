// Multi-tensor fused AdamW over the flat fp32 master buffer.
//
// Semantics of the reference's inner optimiser (node/cli/src/continuous.rs:409-414, Burn AdamW with
// GradientClipping::Norm): each parameter tensor's gradient is clipped to L2 norm <= max_norm
// (coef = min(1, max_norm / (norm + 1e-6))), then
//     p <- p * (1 - lr*wd) - lr * m_hat / (sqrt(v_hat) + eps)
// with bias-corrected first/second moments. A global-norm variant is selected by hp[HP_CLIP_GLOBAL].
//
// Everything the step needs lives on the device (hyper-parameter block, step counter, skip flag), so
// the whole train step can be replayed from a CUDA graph: the host only rewrites hp[HP_LR].
// The update also writes the bf16 compute copy of every parameter used by the GEMMs, and with
// hp[HP_ZERO_GRAD] != 0 it clears every gradient it has read (also on a skipped step), so the next
// step's backward - whose weight-gradient GEMMs accumulate - starts from zero without a separate pass.
#include "common.cuh"

namespace {

enum HP : int {
  HP_LR = 0, HP_B1 = 1, HP_B2 = 2, HP_EPS = 3, HP_WD = 4, HP_BC1 = 5, HP_BC2 = 6, HP_MAXNORM = 7,
  HP_CLIP_GLOBAL = 8, HP_STEP = 9, HP_DO_UPDATE = 10, HP_ZERO_GRAD = 11, HP_COUNT = 16
};

// chunk i covers [cstart[i], cend[i]) of segment cseg[i]
__global__ void seg_sqnorm_kernel(const float* __restrict__ g, const int* __restrict__ cseg,
                                  const long long* __restrict__ cstart, const long long* __restrict__ cend,
                                  float* __restrict__ norms) {
  __shared__ float sh[32];
  const int c = blockIdx.x;
  const long long s = cstart[c], e = cend[c];
  float acc = 0.f;
  long long i = s + threadIdx.x * 4;
  // fast path: 16B-aligned chunk bounds (host guarantees multiples of 4 elements)
  for (; i + 3 < e; i += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(g + i);
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long long j = i; j < e && j < i + 4; ++j) acc += g[j] * g[j];
  float t = block_sum(acc, sh);
  if (threadIdx.x == 0) atomicAdd(norms + cseg[c], t);
}

// Single thread: decide whether to update (finite loss), advance the step and bias corrections.
__global__ void adam_prepare_kernel(float* hp, const float* loss_flag) {
  bool skip = loss_flag && loss_flag[1] != 0.f;
  if (skip) {
    hp[HP_DO_UPDATE] = 0.f;
    return;
  }
  float t = hp[HP_STEP] + 1.f;
  hp[HP_STEP] = t;
  hp[HP_BC1] = 1.f - powf(hp[HP_B1], t);
  hp[HP_BC2] = 1.f - powf(hp[HP_B2], t);
  hp[HP_DO_UPDATE] = 1.f;
}

__global__ void adamw_update_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m,
                                    float* __restrict__ v, __nv_bfloat16* __restrict__ p16, const int* __restrict__ cseg,
                                    const long long* __restrict__ cstart, const long long* __restrict__ cend,
                                    const float* __restrict__ norms, int nseg, const float* __restrict__ hp) {
  const bool upd = hp[HP_DO_UPDATE] != 0.f, zero = hp[HP_ZERO_GRAD] != 0.f;
  const int c = blockIdx.x;
  const long long s = cstart[c], e = cend[c];
  if (!upd) {
    if (zero)
      for (long long i = s + threadIdx.x * 4; i < e; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(g + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  const float lr = hp[HP_LR], b1 = hp[HP_B1], b2 = hp[HP_B2], eps = hp[HP_EPS], wd = hp[HP_WD];
  const float bc1 = hp[HP_BC1], bc2 = hp[HP_BC2], maxn = hp[HP_MAXNORM];
  float coef = 1.f;
  if (maxn > 0.f) {
    float n2;
    if (hp[HP_CLIP_GLOBAL] != 0.f) {
      n2 = 0.f;
      for (int k = 0; k < nseg; ++k) n2 += norms[k];
    } else {
      n2 = norms[cseg[c]];
    }
    coef = fminf(1.f, maxn / (sqrtf(n2) + 1e-6f));
  }
  const float decay = 1.f - lr * wd;
  const float inv_bc1 = 1.f / bc1, inv_sqrt_bc2 = rsqrtf(bc2);
  for (long long i = s + threadIdx.x * 4; i < e; i += blockDim.x * 4) {
    float4 pp = *reinterpret_cast<float4*>(p + i);
    float4 gg = *reinterpret_cast<const float4*>(g + i);
    float4 mm = *reinterpret_cast<float4*>(m + i);
    float4 vv = *reinterpret_cast<float4*>(v + i);
    float* pa = &pp.x; const float* ga = &gg.x; float* ma = &mm.x; float* va = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float gk = ga[k] * coef;
      ma[k] = b1 * ma[k] + (1.f - b1) * gk;
      va[k] = b2 * va[k] + (1.f - b2) * gk * gk;
      float mh = ma[k] * inv_bc1;
      float vh = sqrtf(va[k]) * inv_sqrt_bc2;
      pa[k] = pa[k] * decay - lr * mh / (vh + eps);
    }
    *reinterpret_cast<float4*>(p + i) = pp;
    *reinterpret_cast<float4*>(m + i) = mm;
    *reinterpret_cast<float4*>(v + i) = vv;
    if (zero) *reinterpret_cast<float4*>(g + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (p16) {
      uint2 o;
      o.x = pack_bf16(pp.x, pp.y);
      o.y = pack_bf16(pp.z, pp.w);
      *reinterpret_cast<uint2*>(p16 + i) = o;
    }
  }
}

// fp32 -> bf16 cast of the flat buffer (initial shadow / after a checkpoint swap)
__global__ void cast_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n) {
  for (long long i = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4; i < n;
       i += (long long)gridDim.x * blockDim.x * 4) {
    if (i + 3 < n) {
      float4 a = *reinterpret_cast<const float4*>(x + i);
      uint2 o;
      o.x = pack_bf16(a.x, a.y);
      o.y = pack_bf16(a.z, a.w);
      *reinterpret_cast<uint2*>(y + i) = o;
    } else {
      for (long long j = i; j < n; ++j) y[j] = __float2bfloat16(x[j]);
    }
  }
}

}  // namespace

// Chunk tables (cseg/cstart/cend, `nchunks` entries) are device arrays built once by the host; chunk
// bounds must be multiples of 4 elements and every buffer 16-byte aligned.
DT_API int dt_adamw_step(float* p, float* g, float* m, float* v, void* p16, const int* cseg,
                         const long long* cstart, const long long* cend, int nchunks, float* norms, int nseg,
                         float* hp, const float* loss_flag, cudaStream_t st) {
  DT_CUDA_RET(cudaMemsetAsync(norms, 0, sizeof(float) * nseg, st));
  if (hp) {
    seg_sqnorm_kernel<<<nchunks, 256, 0, st>>>(g, cseg, cstart, cend, norms);
    adam_prepare_kernel<<<1, 1, 0, st>>>(hp, loss_flag);
    adamw_update_kernel<<<nchunks, 256, 0, st>>>(p, g, m, v, reinterpret_cast<__nv_bfloat16*>(p16), cseg, cstart, cend,
                                                 norms, nseg, hp);
  }
  return (int)cudaGetLastError();
}

// Prepare + update only: `norms` already holds the per-segment squared gradient norms (e.g. summed over a
// tensor-parallel group after dt_seg_sqnorm).
DT_API int dt_adamw_apply(float* p, float* g, float* m, float* v, void* p16, const int* cseg,
                          const long long* cstart, const long long* cend, int nchunks, const float* norms, int nseg,
                          float* hp, const float* loss_flag, cudaStream_t st) {
  adam_prepare_kernel<<<1, 1, 0, st>>>(hp, loss_flag);
  adamw_update_kernel<<<nchunks, 256, 0, st>>>(p, g, m, v, reinterpret_cast<__nv_bfloat16*>(p16), cseg, cstart, cend,
                                               norms, nseg, hp);
  return (int)cudaGetLastError();
}

DT_API int dt_seg_sqnorm(const float* g, const int* cseg, const long long* cstart, const long long* cend, int nchunks,
                         float* norms, int nseg, cudaStream_t st) {
  DT_CUDA_RET(cudaMemsetAsync(norms, 0, sizeof(float) * nseg, st));
  seg_sqnorm_kernel<<<nchunks, 256, 0, st>>>(g, cseg, cstart, cend, norms);
  return (int)cudaGetLastError();
}

DT_API int dt_cast_bf16(const float* x, void* y, long long n, cudaStream_t st) {
  long long blocks = (n / 4 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  cast_bf16_kernel<<<(int)blocks, 256, 0, st>>>(x, reinterpret_cast<__nv_bfloat16*>(y), n);
  return (int)cudaGetLastError();
}
