// QKV bias + rotary embedding (rotate-half form, reference model.rs:66-122) applied in place on the
// fused QKV GEMM output, and its backward (inverse rotation + bias gradient).
//
// Row m of qkv = [q heads (nh*d) | k heads (nkv*d) | v heads (nkv*d)], position t = m % T.
// Pair (i, i+d/2) of a rotated head: out_i = x_i cos - x_{i+d/2} sin ; out_{i+d/2} = x_i sin + x_{i+d/2} cos.
// cos/sin tables are [T, d/2] fp32, built on the host with the reference's fp32 formula.
#include "common.cuh"

namespace {

// Block = (items, ry <= RY_MAX) threads over ROWS_F (forward) / ROWS_B (backward) rows; ry rows are
// processed in parallel. The backward reduces the bias gradient over the block's rows through shared
// memory and issues one atomic per column per block (64 rows), not per 16 rows and thread.
constexpr int RY_MAX = 4, ROWS_F = 16, ROWS_B = 64;

// Work items per row, in units of 8 elements: P8 = (nh+nkv) * d/16 rotation groups (8 pairs each),
// then V8 = nkv * d/8 groups of v elements.
__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
  uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 f = unpack_bf16(w[k]);
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

template <bool BWD>
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ bias, float* __restrict__ dbias,
                            const float* __restrict__ cosT, const float* __restrict__ sinT, int M, int T, int nh,
                            int nkv, int d) {
  const int half = d / 2, W_ = (nh + 2 * nkv) * d;
  const int g_per_head = half / 8;
  const int P8 = (nh + nkv) * g_per_head, V8 = nkv * d / 8, items = P8 + V8;
  const int vbase = (nh + nkv) * d;
  const int j = threadIdx.x, y = threadIdx.y, RY = blockDim.y;  // one item per thread (blockDim.x >= items, host-checked)
  const bool active = j < items;
  int c0 = 0, c1 = -1, i0 = 0;
  if (!active) {
  } else if (j < P8) {
    int head = j / g_per_head, g = j - head * g_per_head;
    i0 = g * 8;
    c0 = head * d + i0;
    c1 = c0 + half;
  } else {
    c0 = vbase + (j - P8) * 8;
  }
  float acc0[8], acc1[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc0[k] = acc1[k] = 0.f;
  float b0[8], b1[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    b0[k] = (!BWD && bias && active) ? bias[c0 + k] : 0.f;
    b1[k] = (!BWD && bias && c1 >= 0) ? bias[c1 + k] : 0.f;
  }
  const int rows = BWD ? ROWS_B : ROWS_F;
  const long long r0 = (long long)blockIdx.x * rows;
  // the next row's two 16-byte groups are loaded (kept packed, 8 registers) before this row is worked on
  uint4 na = make_uint4(0, 0, 0, 0), nb = na;
  auto fetch = [&](long long row) {
    const __nv_bfloat16* q = qkv + row * W_;
    na = *reinterpret_cast<const uint4*>(q + c0);
    if (c1 >= 0) nb = *reinterpret_cast<const uint4*>(q + c1);
  };
  if (active && r0 + y < M && y < rows) fetch(r0 + y);
  for (int rr = y; rr < rows && active; rr += RY) {
    const long long row = r0 + rr;
    if (row >= M) break;
    const int t = (int)(row % T);
    __nv_bfloat16* p = qkv + row * W_;
    const uint4 ua = na, ub = nb;
    if (rr + RY < rows && row + RY < M) fetch(row + RY);
    float a[8];
    unpack8(ua, a);
    if (c1 < 0) {
      if (BWD) {
#pragma unroll
        for (int k = 0; k < 8; ++k) acc0[k] += a[k];
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] += b0[k];
        store8(p + c0, a);
      }
      continue;
    }
    float b[8];
    unpack8(ub, b);
    const float4* cp = reinterpret_cast<const float4*>(cosT + (long long)t * half + i0);
    const float4* sp = reinterpret_cast<const float4*>(sinT + (long long)t * half + i0);
    float4 ca = cp[0], cb = cp[1], sa = sp[0], sb = sp[1];
    float cs[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
    float sn[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
    float o0[8], o1[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (BWD) {  // inverse rotation of the incoming gradient
        o0[k] = a[k] * cs[k] + b[k] * sn[k];
        o1[k] = -a[k] * sn[k] + b[k] * cs[k];
        acc0[k] += o0[k];
        acc1[k] += o1[k];
      } else {
        float x = a[k] + b0[k], y = b[k] + b1[k];
        o0[k] = x * cs[k] - y * sn[k];
        o1[k] = x * sn[k] + y * cs[k];
      }
    }
    store8(p + c0, o0);
    store8(p + c1, o1);
  }
  if (BWD && dbias) {
    extern __shared__ float red[];  // [RY][blockDim.x][16]
    float* mine = red + ((size_t)y * blockDim.x + j) * 16;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mine[k] = acc0[k];
      mine[8 + k] = acc1[k];
    }
    __syncthreads();
    if (y == 0 && active) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        float t = 0.f;
        for (int yy = 0; yy < RY; ++yy) t += red[((size_t)yy * blockDim.x + j) * 16 + k];
        if (k < 8) atomicAdd(dbias + c0 + k, t);
        else if (c1 >= 0) atomicAdd(dbias + c1 + k - 8, t);
      }
    }
  }
}

}  // namespace

static int rope_launch(bool bwd, void* qkv, const float* bias, float* dbias, const float* cosT, const float* sinT,
                       int M, int T, int nh, int nkv, int d, cudaStream_t st) {
  if (d % 16) return -10;
  int items = (nh + nkv) * (d / 16) + nkv * d / 8;
  int th = ((items + 31) / 32) * 32;
  if (th > 1024) return -11;
  int ry = RY_MAX;  // row lanes: the block stays <= 1024 threads and its reduction buffer <= 48 KB
  while (ry > 1 && (th * ry > 1024 || sizeof(float) * 16 * th * ry > 48 * 1024)) ry /= 2;
  if (th * ry > 1024 || sizeof(float) * 16 * th * ry > 48 * 1024) return -11;
  const int rows = bwd ? ROWS_B : ROWS_F;
  int blocks = (M + rows - 1) / rows;
  auto p = reinterpret_cast<__nv_bfloat16*>(qkv);
  dim3 blk(th, ry);
  if (bwd) {
    size_t sm = sizeof(float) * 16 * th * ry;
    rope_kernel<true><<<blocks, blk, sm, st>>>(p, nullptr, dbias, cosT, sinT, M, T, nh, nkv, d);
  } else {
    rope_kernel<false><<<blocks, blk, 0, st>>>(p, bias, nullptr, cosT, sinT, M, T, nh, nkv, d);
  }
  return (int)cudaGetLastError();
}

DT_API int dt_rope_fwd(void* qkv, const float* bias, const float* cosT, const float* sinT, int M, int T, int nh,
                       int nkv, int d, cudaStream_t st) {
  return rope_launch(false, qkv, bias, nullptr, cosT, sinT, M, T, nh, nkv, d, st);
}

DT_API int dt_rope_bwd(void* dqkv, float* dbias, const float* cosT, const float* sinT, int M, int T, int nh, int nkv,
                       int d, cudaStream_t st) {
  return rope_launch(true, dqkv, nullptr, dbias, cosT, sinT, M, T, nh, nkv, d, st);
}
