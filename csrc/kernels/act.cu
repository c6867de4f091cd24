// SwiGLU activation (reference model.rs:292-296: down(silu(x Wg) * (x Wu))) forward/backward on the
// fused gate|up GEMM output, and the softmax cross-entropy over the tied LM-head logits
// (model.rs:804-811: -mean(log_softmax(z)[target])) with the logits gradient written in place.
#include "common.cuh"

namespace {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// gu: [M, 2F] (gate cols [0,F), up cols [F,2F)), h: [M, F]. 8 bf16 per thread-iteration.
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, long long M,
                                  int F) {
  long long n8 = M * (long long)(F / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    long long row = i / (F / 8);
    int c = (int)(i - row * (F / 8)) * 8;
    uint4 g = *reinterpret_cast<const uint4*>(gu + row * 2 * F + c);
    uint4 u = *reinterpret_cast<const uint4*>(gu + row * 2 * F + F + c);
    uint32_t gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w}, o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 a = unpack_bf16(gg[k]), b = unpack_bf16(uu[k]);
      o[k] = pack_bf16(a.x * sigmoidf_(a.x) * b.x, a.y * sigmoidf_(a.y) * b.y);
    }
    *reinterpret_cast<uint4*>(h + row * F + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// dgu[:, gate] = dh * u * silu'(g) ; dgu[:, up] = dh * silu(g).  dgu may alias gu.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* gu,
                                  __nv_bfloat16* dgu, long long M, int F) {
  long long n8 = M * (long long)(F / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    long long row = i / (F / 8);
    int c = (int)(i - row * (F / 8)) * 8;
    uint4 g = *reinterpret_cast<const uint4*>(gu + row * 2 * F + c);
    uint4 u = *reinterpret_cast<const uint4*>(gu + row * 2 * F + F + c);
    uint4 d = *reinterpret_cast<const uint4*>(dh + row * F + c);
    uint32_t gg[4] = {g.x, g.y, g.z, g.w}, uu[4] = {u.x, u.y, u.z, u.w}, dd[4] = {d.x, d.y, d.z, d.w};
    uint32_t og[4], ou[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 a = unpack_bf16(gg[k]), b = unpack_bf16(uu[k]), e = unpack_bf16(dd[k]);
      float s0 = sigmoidf_(a.x), s1 = sigmoidf_(a.y);
      float silu0 = a.x * s0, silu1 = a.y * s1;
      float ds0 = s0 * (1.f + a.x * (1.f - s0)), ds1 = s1 * (1.f + a.y * (1.f - s1));
      og[k] = pack_bf16(e.x * b.x * ds0, e.y * b.y * ds1);
      ou[k] = pack_bf16(e.x * silu0, e.y * silu1);
    }
    *reinterpret_cast<uint4*>(dgu + row * 2 * F + c) = make_uint4(og[0], og[1], og[2], og[3]);
    *reinterpret_cast<uint4*>(dgu + row * 2 * F + F + c) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
  }
}

// One block per row of logits [rows, V] (bf16). loss_row[r] = lse - z[target]; logits are replaced by
// grad_scale * (softmax - onehot(target)).  Target of row r (global row r0 + r) = ids[b*S + t + 1].
__global__ void ce_fwd_bwd_kernel(__nv_bfloat16* __restrict__ logits, long long ld, const int* __restrict__ ids,
                                  int T, int S, long long r0, float* __restrict__ loss_row, int V,
                                  float grad_scale) {
  __shared__ float sh[32];
  __shared__ float sh_m[32];
  const long long r = blockIdx.x;
  const long long grow = r0 + r;
  const long long b = grow / T, t = grow - b * T;
  const int tgt = ids[b * S + t + 1];
  __nv_bfloat16* z = logits + r * ld;
  // pass 1: online max / sum-exp per thread over 8-wide vectors
  float m = -INFINITY, s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 q = *reinterpret_cast<const uint4*>(z + c);
    uint32_t qq[4] = {q.x, q.y, q.z, q.w};
    float v[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16(qq[k]);
      v[2 * k] = f.x;
      v[2 * k + 1] = f.y;
    }
    float lm = v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) lm = fmaxf(lm, v[k]);
    float nm = fmaxf(m, lm);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += __expf(v[k] - nm);
    s = s * __expf(m - nm) + acc;
    m = nm;
  }
  // block combine (max then rescaled sum)
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float wm = warp_max(m);
  float ws = warp_sum(m == -INFINITY ? 0.f : s * __expf(m - wm));
  if (lane == 0) { sh_m[wid] = wm; sh[wid] = ws; }
  __syncthreads();
  int nw = blockDim.x >> 5;
  if (wid == 0) {
    float mm = lane < nw ? sh_m[lane] : -INFINITY;
    float ss = lane < nw ? sh[lane] : 0.f;
    float gm = warp_max(mm);
    float gs = warp_sum((lane < nw && mm != -INFINITY) ? ss * __expf(mm - gm) : 0.f);
    if (lane == 0) { sh_m[0] = gm; sh[0] = gs; }
  }
  __syncthreads();
  const float gmax = sh_m[0], gsum = sh[0];
  const float lse = gmax + __logf(gsum);
  if (threadIdx.x == 0) loss_row[r] = lse - __bfloat162float(z[tgt]);
  __syncthreads();
  const float inv = 1.f / gsum;
  // pass 2: gradient in place
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 q = *reinterpret_cast<const uint4*>(z + c);
    uint32_t qq[4] = {q.x, q.y, q.z, q.w}, o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16(qq[k]);
      float p0 = __expf(f.x - gmax) * inv, p1 = __expf(f.y - gmax) * inv;
      if (c + 2 * k == tgt) p0 -= 1.f;
      if (c + 2 * k + 1 == tgt) p1 -= 1.f;
      o[k] = pack_bf16(p0 * grad_scale, p1 * grad_scale);
    }
    *reinterpret_cast<uint4*>(z + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Cross-entropy from the LM-head GEMM's fp32 softmax statistics (dt_gemm_logits_lse): one block per row
// combines the row's `np` partial (max, sum exp) pairs into the log-sum-exp, writes
// loss_row[r] = lse - target logit (both fp32), then replaces the bf16 logits of the row with
// grad_scale * (softmax - onehot(target)) in one read + write pass. With per-row weights `row_w`
// (indexed like the rows of `ids`, i.e. by r0 + r; may be negative) the row's gradient is scaled by its
// weight as well: a loss mask (fine-tuning on response tokens) or a signed preference coefficient. The
// loss row stays the unweighted cross-entropy; dt_loss_reduce applies the same weights.
__global__ void ce_lse_bwd_kernel(__nv_bfloat16* __restrict__ logits, long long ld, const float2* __restrict__ part,
                                  int np, long long rows, const float* __restrict__ tgt_logit,
                                  const int* __restrict__ ids, int T, int S, long long r0,
                                  float* __restrict__ loss_row, int V, float grad_scale,
                                  const float* __restrict__ row_w) {
  __shared__ float sh[32];
  __shared__ float sh_m[32];
  const long long r = blockIdx.x;
  const long long grow = r0 + r;
  const long long b = grow / T, t = grow - b * T;
  const int tgt = ids[b * S + t + 1];
  if (row_w) grad_scale *= row_w[grow];
  float m = -INFINITY, s = 0.f;
  for (int k = threadIdx.x; k < np; k += blockDim.x) {
    const float2 p = part[(long long)k * rows + r];
    if (p.x == -INFINITY) continue;
    const float nm = fmaxf(m, p.x);
    s = s * __expf(m - nm) + p.y * __expf(p.x - nm);
    m = nm;
  }
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float wm = warp_max(m);
  float ws = warp_sum(m == -INFINITY ? 0.f : s * __expf(m - wm));
  if (lane == 0) { sh_m[wid] = wm; sh[wid] = ws; }
  __syncthreads();
  int nw = blockDim.x >> 5;
  if (wid == 0) {
    float mm = lane < nw ? sh_m[lane] : -INFINITY;
    float ss = lane < nw ? sh[lane] : 0.f;
    float gm = warp_max(mm);
    float gs = warp_sum((lane < nw && mm != -INFINITY) ? ss * __expf(mm - gm) : 0.f);
    if (lane == 0) { sh_m[0] = gm; sh[0] = gs; }
  }
  __syncthreads();
  const float lse = sh_m[0] + __logf(sh[0]);
  if (threadIdx.x == 0) loss_row[r] = lse - tgt_logit[r];
  __nv_bfloat16* z = logits + r * ld;
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 q = *reinterpret_cast<const uint4*>(z + c);
    uint32_t qq[4] = {q.x, q.y, q.z, q.w}, o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16(qq[k]);
      float p0 = __expf(f.x - lse), p1 = __expf(f.y - lse);
      if (c + 2 * k == tgt) p0 -= 1.f;
      if (c + 2 * k + 1 == tgt) p1 -= 1.f;
      o[k] = pack_bf16(p0 * grad_scale, p1 * grad_scale);
    }
    *reinterpret_cast<uint4*>(z + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// out[0] = sum(w[i] * loss_row[i], i < n) * scale, w = 1 without weights (single block); out[1] = 1 if
// non-finite; out[2] += out[0] and out[3] += 1 when finite (running round sums read at push time).
__global__ void loss_reduce_kernel(const float* __restrict__ loss_row, long long n, float scale, float* out,
                                   const float* __restrict__ w) {
  __shared__ float sh[32];
  float s = 0.f;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) {
    // a zero weight drops its row even when that row's loss is not finite (padding)
    if (w) s += w[i] != 0.f ? w[i] * loss_row[i] : 0.f;
    else s += loss_row[i];
  }
  float tot = block_sum(s, sh);
  if (threadIdx.x == 0) {
    float l = tot * scale;
    out[0] = l;
    out[1] = isfinite(l) ? 0.f : 1.f;
    if (isfinite(l)) {
      out[2] += l;
      out[3] += 1.f;
    }
  }
}

int grid_for(long long n, int th) {
  long long b = (n + th - 1) / th;
  if (b > 148 * 16) b = 148 * 16;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

DT_API int dt_swiglu_fwd(const void* gu, void* h, long long M, int F, cudaStream_t st) {
  if (F % 8) return -10;
  long long n = M * (F / 8);
  swiglu_fwd_kernel<<<grid_for(n, 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(gu),
                                                       reinterpret_cast<__nv_bfloat16*>(h), M, F);
  return (int)cudaGetLastError();
}

DT_API int dt_swiglu_bwd(const void* dh, const void* gu, void* dgu, long long M, int F, cudaStream_t st) {
  if (F % 8) return -10;
  long long n = M * (F / 8);
  swiglu_bwd_kernel<<<grid_for(n, 256), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dh),
                                                       reinterpret_cast<const __nv_bfloat16*>(gu),
                                                       reinterpret_cast<__nv_bfloat16*>(dgu), M, F);
  return (int)cudaGetLastError();
}

DT_API int dt_ce_fwd_bwd(void* logits, long long ld, const int* ids, int T, int S, long long r0, long long rows,
                         float* loss_row, int V, float grad_scale, cudaStream_t st) {
  if (V % 8 || ld % 8) return -10;
  ce_fwd_bwd_kernel<<<(unsigned)rows, 512, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld, ids, T, S, r0,
                                                    loss_row, V, grad_scale);
  return (int)cudaGetLastError();
}

DT_API int dt_loss_reduce(const float* loss_row, long long n, float scale, float* out, const float* w,
                          cudaStream_t st) {
  loss_reduce_kernel<<<1, 1024, 0, st>>>(loss_row, n, scale, out, w);
  return (int)cudaGetLastError();
}

DT_API int dt_ce_lse_bwd(void* logits, long long ld, const void* part, int np, long long rows, const float* tgt_logit,
                         const int* ids, int T, int S, long long r0, float* loss_row, int V, float grad_scale,
                         const float* row_w, cudaStream_t st) {
  if (V % 8 || ld % 8 || rows <= 0) return rows <= 0 ? 0 : -10;
  ce_lse_bwd_kernel<<<(unsigned)rows, 512, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(logits), ld,
                                                    reinterpret_cast<const float2*>(part), np, rows, tgt_logit, ids,
                                                    T, S, r0, loss_row, V, grad_scale, row_w);
  return (int)cudaGetLastError();
}
