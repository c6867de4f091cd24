// QKV bias + rotary embedding (rotate-half form, reference model.rs:66-122) applied in place on the
// fused QKV GEMM output, and its backward (inverse rotation + bias gradient).
//
// Row m of qkv = [q heads (nh*d) | k heads (nkv*d) | v heads (nkv*d)], position t = m % T.
// Pair (i, i+d/2) of a rotated head: out_i = x_i cos - x_{i+d/2} sin ; out_{i+d/2} = x_i sin + x_{i+d/2} cos.
// cos/sin tables are [T, d/2] fp32, built on the host with the reference's fp32 formula.
#include "common.cuh"

namespace {

constexpr int ROWS = 16;
constexpr int MAX_ITEMS = 8;

// Work item j < P: rotation pair; j >= P: v element.  P = (nh+nkv)*d/2.
__device__ __forceinline__ void item_cols(int j, int P, int half, int d, int vbase, int& c0, int& c1) {
  if (j < P) {
    int head = j / half, i = j - head * half;
    c0 = head * d + i;
    c1 = c0 + half;
  } else {
    c0 = vbase + (j - P);
    c1 = -1;
  }
}

__global__ void rope_fwd_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ bias,
                                const float* __restrict__ cosT, const float* __restrict__ sinT, int M, int T, int nh,
                                int nkv, int d) {
  const int half = d / 2, W_ = (nh + 2 * nkv) * d;
  const int P = (nh + nkv) * half, items = P + nkv * d, vbase = (nh + nkv) * d;
  const int r0 = blockIdx.x * ROWS;
  for (int rr = 0; rr < ROWS; ++rr) {
    long long row = r0 + rr;
    if (row >= M) break;
    int t = (int)(row % T);
    __nv_bfloat16* p = qkv + row * W_;
    for (int j = threadIdx.x; j < items; j += blockDim.x) {
      int c0, c1;
      item_cols(j, P, half, d, vbase, c0, c1);
      float a = __bfloat162float(p[c0]) + (bias ? bias[c0] : 0.f);
      if (c1 >= 0) {
        float b = __bfloat162float(p[c1]) + (bias ? bias[c1] : 0.f);
        int i = c0 % d;
        float cs = cosT[t * half + i], sn = sinT[t * half + i];
        p[c0] = __float2bfloat16(a * cs - b * sn);
        p[c1] = __float2bfloat16(a * sn + b * cs);
      } else {
        p[c0] = __float2bfloat16(a);
      }
    }
  }
}

__global__ void rope_bwd_kernel(__nv_bfloat16* __restrict__ dqkv, float* __restrict__ dbias,
                                const float* __restrict__ cosT, const float* __restrict__ sinT, int M, int T, int nh,
                                int nkv, int d) {
  const int half = d / 2, W_ = (nh + 2 * nkv) * d;
  const int P = (nh + nkv) * half, items = P + nkv * d, vbase = (nh + nkv) * d;
  float acc0[MAX_ITEMS], acc1[MAX_ITEMS];
#pragma unroll
  for (int k = 0; k < MAX_ITEMS; ++k) acc0[k] = acc1[k] = 0.f;
  const int r0 = blockIdx.x * ROWS;
  for (int rr = 0; rr < ROWS; ++rr) {
    long long row = r0 + rr;
    if (row >= M) break;
    int t = (int)(row % T);
    __nv_bfloat16* p = dqkv + row * W_;
#pragma unroll
    for (int k = 0; k < MAX_ITEMS; ++k) {
      int j = threadIdx.x + k * blockDim.x;
      if (j >= items) break;
      int c0, c1;
      item_cols(j, P, half, d, vbase, c0, c1);
      float ga = __bfloat162float(p[c0]);
      if (c1 >= 0) {
        float gb = __bfloat162float(p[c1]);
        int i = c0 % d;
        float cs = cosT[t * half + i], sn = sinT[t * half + i];
        float da = ga * cs + gb * sn, db = -ga * sn + gb * cs;
        p[c0] = __float2bfloat16(da);
        p[c1] = __float2bfloat16(db);
        acc0[k] += da;
        acc1[k] += db;
      } else {
        acc0[k] += ga;
      }
    }
  }
  if (!dbias) return;
#pragma unroll
  for (int k = 0; k < MAX_ITEMS; ++k) {
    int j = threadIdx.x + k * blockDim.x;
    if (j >= items) break;
    int c0, c1;
    item_cols(j, P, half, d, vbase, c0, c1);
    atomicAdd(dbias + c0, acc0[k]);
    if (c1 >= 0) atomicAdd(dbias + c1, acc1[k]);
  }
}

}  // namespace

DT_API int dt_rope_fwd(void* qkv, const float* bias, const float* cosT, const float* sinT, int M, int T, int nh,
                       int nkv, int d, cudaStream_t st) {
  if (d % 2) return -10;
  int blocks = (M + ROWS - 1) / ROWS;
  rope_fwd_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(qkv), bias, cosT, sinT, M, T, nh, nkv, d);
  return (int)cudaGetLastError();
}

DT_API int dt_rope_bwd(void* dqkv, float* dbias, const float* cosT, const float* sinT, int M, int T, int nh, int nkv,
                       int d, cudaStream_t st) {
  int items = (nh + nkv) * d / 2 + nkv * d;
  int th = (items + MAX_ITEMS - 1) / MAX_ITEMS;
  th = ((th + 31) / 32) * 32;
  if (th < 128) th = items < 128 ? ((items + 31) / 32) * 32 : 128;
  if (th > 1024) return -11;
  int blocks = (M + ROWS - 1) / ROWS;
  rope_bwd_kernel<<<blocks, th, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(dqkv), dbias, cosT, sinT, M, T, nh, nkv, d);
  return (int)cudaGetLastError();
}
