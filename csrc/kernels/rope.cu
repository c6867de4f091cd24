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
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
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
  for (int rr = y; rr < rows && active; rr += RY) {
    const long long row = r0 + rr;
    if (row >= M) break;
    const int t = (int)(row % T);
    __nv_bfloat16* p = qkv + row * W_;
    float a[8];
    load8(p + c0, a);
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
    load8(p + c1, b);
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

namespace {
// ───────────── RoPE backward, streaming form: inverse rotation in place + bias-gradient partials ─────────────
// Block = 8 warps over RB rows; a warp takes every 8th row, 4 rows per step, one 256-column window of the
// row per pass (lane l: columns 8l..8l+7). The rotation partner of a q / k column lies D/2 columns away,
// which is lane l ^ (D/16) of the same window (windows start on head boundaries: 256 % D == 0).
// Column sums of the rotated-back rows go to part[block][W] (no atomics); dt_rope_bwd_stream's second
// kernel adds them into dbias.
constexpr int RB = 128;
template <int D>
__global__ void __launch_bounds__(256) rope_bwd_stream_kernel(
    __nv_bfloat16* __restrict__ g, const float* __restrict__ cosT, const float* __restrict__ sinT, long long M,
    int T, int W, int rot_cols, float* __restrict__ part) {
  __shared__ float red[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r0 = (long long)blockIdx.x * RB;
  const long long r1 = r0 + RB < M ? r0 + RB : M;
  constexpr int PL = D / 16;
  for (int w0 = 0; w0 < W; w0 += 256) {
    const int col = w0 + lane * 8;
    const bool rot = col < rot_cols;
    const bool first = (col % D) < D / 2;
    const int j = (col % D) % (D / 2);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.f;
    for (long long rb = r0 + warp; rb < r1; rb += 32) {
      float v[4][8];
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long row = rb + 8 * u;
        raw[u] = row < r1 ? *reinterpret_cast<const uint4*>(g + row * W + col) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long row = rb + 8 * u;
        const uint32_t w4[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
        float a[8], b[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16(w4[k]);
          a[2 * k] = f.x;
          a[2 * k + 1] = f.y;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) b[k] = __shfl_xor_sync(0xffffffffu, a[k], PL);
        if (row < r1 && rot) {
          const int t = (int)(row % T);
          const float4* cp = reinterpret_cast<const float4*>(cosT + (long long)t * (D / 2) + j);
          const float4* sp = reinterpret_cast<const float4*>(sinT + (long long)t * (D / 2) + j);
          const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
          const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
          for (int k = 0; k < 8; ++k)  // first half: a = grad at j, b = grad at j + D/2; second: swapped
            v[u][k] = first ? (a[k] * cs[k] + b[k] * sn[k]) : (a[k] * cs[k] - b[k] * sn[k]);
          uint4 o;
          o.x = pack_bf16(v[u][0], v[u][1]);
          o.y = pack_bf16(v[u][2], v[u][3]);
          o.z = pack_bf16(v[u][4], v[u][5]);
          o.w = pack_bf16(v[u][6], v[u][7]);
          *reinterpret_cast<uint4*>(g + row * W + col) = o;
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) v[u][k] = row < r1 ? a[k] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] += v[u][k];
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) red[warp][lane * 8 + k] = acc[k];
    __syncthreads();
    {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += red[w][threadIdx.x];
      if (w0 + threadIdx.x < W) part[(long long)blockIdx.x * W + w0 + threadIdx.x] = t;
    }
    __syncthreads();
  }
}

__global__ void add_partials_kernel(const float* __restrict__ part, int nblocks, int W, float* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= W) return;
  float t = 0.f;
  for (int b = 0; b < nblocks; ++b) t += part[(long long)b * W + c];
  out[c] += t;
}
}  // namespace

DT_API long long dt_rope_bwd_stream_scratch(long long M, int W) { return ((M + RB - 1) / RB) * (long long)W; }


// In-place inverse rotation of the q / k heads of dqkv [M, W] (the gradient of the rotated projection
// becomes that of the unrotated one) and dbias += its column sums (null dbias: rotation only, the
// partials are still formed). `scratch`: dt_rope_bwd_stream_scratch(M, W) floats. d = 64 / 128 and
// W a multiple of 256; other shapes use dt_rope_bwd.
DT_API int dt_rope_bwd_stream(void* dqkv, float* dbias, const float* cosT, const float* sinT, long long M, int T,
                              int nh, int nkv, int d, float* scratch, cudaStream_t st) {
  const int W = (nh + 2 * nkv) * d;
  if ((d != 64 && d != 128) || (W % 256) || !scratch || (reinterpret_cast<uintptr_t>(dqkv) & 15)) return -10;
  if (M <= 0) return 0;
  const int nb = (int)((M + RB - 1) / RB);
  auto p = reinterpret_cast<__nv_bfloat16*>(dqkv);
  const int rot = (nh + nkv) * d;
  if (d == 64) rope_bwd_stream_kernel<64><<<nb, 256, 0, st>>>(p, cosT, sinT, M, T, W, rot, scratch);
  else rope_bwd_stream_kernel<128><<<nb, 256, 0, st>>>(p, cosT, sinT, M, T, W, rot, scratch);
  DT_CUDA_RET(cudaGetLastError());
  if (dbias) add_partials_kernel<<<(W + 255) / 256, 256, 0, st>>>(scratch, nb, W, dbias);
  return (int)cudaGetLastError();
}

namespace {
// ───────────── bias gradient of the QKV projection: column sums of a bf16 [M, W] matrix ─────────────
// out[c] += sum_r x[r, c] (fp32). Block = 32 column groups of 8 columns x 8 row lanes over CS_ROWS rows;
// one atomic per column per block.
constexpr int CS_ROWS = 512;
__global__ void colsum_bf16_kernel(const __nv_bfloat16* __restrict__ x, long long M, int W, float* __restrict__ out) {
  __shared__ float red[8][32][9];
  const int cgp = blockIdx.x * 32 + threadIdx.x;  // column group of 8
  const int c0 = cgp * 8;
  const long long r0 = (long long)blockIdx.y * CS_ROWS;
  float acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  if (c0 < W) {
    const long long r1 = r0 + CS_ROWS < M ? r0 + CS_ROWS : M;
    for (long long r = r0 + threadIdx.y; r < r1; r += 8) {
      float v[8];
      load8(x + r * W + c0, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += v[k];
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) red[threadIdx.y][threadIdx.x][k] = acc[k];
  __syncthreads();
  if (threadIdx.y == 0 && c0 < W) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float t = 0.f;
#pragma unroll
      for (int y = 0; y < 8; ++y) t += red[y][threadIdx.x][k];
      atomicAdd(out + c0 + k, t);
    }
  }
}
}  // namespace

DT_API int dt_colsum_bf16(const void* x, long long M, int W, float* out, cudaStream_t st) {
  if ((W % 8) || (reinterpret_cast<uintptr_t>(x) & 15)) return -10;
  if (M <= 0) return 0;
  dim3 grid((unsigned)((W / 8 + 31) / 32), (unsigned)((M + CS_ROWS - 1) / CS_ROWS));
  colsum_bf16_kernel<<<grid, dim3(32, 8), 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), M, W, out);
  return (int)cudaGetLastError();
}
