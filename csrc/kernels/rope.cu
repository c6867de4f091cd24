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
// memory; the block's column sums then go either to a scratch row of their own (part[block][W], summed
// by rope_bias_reduce_kernel) or, without scratch, as one atomic per column per block. Measured on the
// tiny QKV (32736 x 1280): the atomics - 512 blocks on the same 1280 addresses - took about half of
// the kernel's 65 us, and halving ROWS_B (twice the atomics) cost a further 35 us.
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
                            float* __restrict__ part, const float* __restrict__ cosT, const float* __restrict__ sinT,
                            int M, int T, int nh, int nkv, int d) {
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
  if (BWD && (dbias || part)) {
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
        const int col = k < 8 ? c0 + k : (c1 >= 0 ? c1 + k - 8 : -1);
        if (col < 0) continue;
        if (part) part[(size_t)blockIdx.x * W_ + col] = t;  // every column has exactly one owner per block
        else atomicAdd(dbias + col, t);
      }
    }
  }
}

// dbias[c] += sum over the nblk rows of part[., c]: block = 32 columns x 32 row lanes, each lane summing
// every 32nd row (independent L2 loads), then a shared-memory reduction over the lanes.
__global__ void __launch_bounds__(1024) rope_bias_reduce_kernel(const float* __restrict__ part, int nblk, int W,
                                                                float* __restrict__ dbias) {
  __shared__ float red[32][33];
  const int c = blockIdx.x * 32 + threadIdx.x;
  float t = 0.f;
  if (c < W)
    for (int b = threadIdx.y; b < nblk; b += 32) t += part[(size_t)b * W + c];
  red[threadIdx.y][threadIdx.x] = t;
  __syncthreads();
  if (threadIdx.y == 0 && c < W) {
    float s = 0.f;
#pragma unroll 8
    for (int yy = 0; yy < 32; ++yy) s += red[yy][threadIdx.x];
    dbias[c] += s;
  }
}

}  // namespace

static int rope_launch(bool bwd, void* qkv, const float* bias, float* dbias, float* part, const float* cosT,
                       const float* sinT, int M, int T, int nh, int nkv, int d, cudaStream_t st) {
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
    float* pp = dbias ? part : nullptr;
    rope_kernel<true><<<blocks, blk, sm, st>>>(p, nullptr, dbias, pp, cosT, sinT, M, T, nh, nkv, d);
    if (pp) {
      const int W_ = (nh + 2 * nkv) * d;
      rope_bias_reduce_kernel<<<(W_ + 31) / 32, dim3(32, 32), 0, st>>>(pp, blocks, W_, dbias);
    }
  } else {
    rope_kernel<false><<<blocks, blk, 0, st>>>(p, bias, nullptr, nullptr, cosT, sinT, M, T, nh, nkv, d);
  }
  return (int)cudaGetLastError();
}

// Floats of scratch dt_rope_bwd needs for the two-level bias reduction of M rows: one row of W per block.
DT_API long long dt_rope_bwd_scratch(int M, int nh, int nkv, int d) {
  return (long long)((M + ROWS_B - 1) / ROWS_B) * (nh + 2 * nkv) * d;
}

DT_API int dt_rope_fwd(void* qkv, const float* bias, const float* cosT, const float* sinT, int M, int T, int nh,
                       int nkv, int d, cudaStream_t st) {
  return rope_launch(false, qkv, bias, nullptr, nullptr, cosT, sinT, M, T, nh, nkv, d, st);
}

// part: scratch of dt_rope_bwd_scratch(M, ...) floats, or null (one atomic per column and block instead).
DT_API int dt_rope_bwd(void* dqkv, float* dbias, float* part, const float* cosT, const float* sinT, int M, int T,
                       int nh, int nkv, int d, cudaStream_t st) {
  return rope_launch(true, dqkv, nullptr, dbias, part, cosT, sinT, M, T, nh, nkv, d, st);
}
