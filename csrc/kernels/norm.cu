// RMSNorm forward/backward with the residual add, the embedding gather and the tied-head output
// scale fused in, plus the embedding-gradient scatter-add.
//
// Reference semantics (core/model/src/model.rs:51-59): y = x * rsqrt(mean(x^2) + eps) * w, computed
// in fp32. The residual stream is kept in fp32; the normalised output feeds the GEMMs in bf16.
//
// Layout: rows = B*T tokens, H columns; token row m = b*T + t reads token ids[b*S + t] (the model
// input drops the last token of each length-S sequence, model.rs:791-794).
#include "common.cuh"

namespace {

constexpr int ROWS_BWD = 32;  // rows per block in the backward (amortises dw atomics)

// One block per row, each thread owns VPT float4 column groups.
template <int VPT>
__global__ void add_rmsnorm_fwd_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ br,
                                       const float* __restrict__ emb, const int* __restrict__ ids, int T, int S,
                                       const float* __restrict__ w, const float* __restrict__ scale,
                                       float* __restrict__ out_resid, __nv_bfloat16* __restrict__ y,
                                       float* __restrict__ rstd_out, int H, float eps,
                                       const __nv_bfloat16* br2, PeerWait pw) {
  __shared__ float sh[32];
  __shared__ int sh_ok;
  const long long row = blockIdx.x;
  if (!peer_wait_begin(pw, &sh_ok)) {
    peer_wait_end(pw);
    return;
  }
  const float* src;
  if (emb) {
    long long b = row / T, t = row - b * T;
    src = emb + (long long)ids[b * S + t] * H;
  } else {
    src = x + row * H;
  }
  float4 v[VPT];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    int c = (threadIdx.x + i * blockDim.x) * 4;
    if (c < H) {
      float4 a = *reinterpret_cast<const float4*>(src + c);
      if (br) {
        uint2 bb = *reinterpret_cast<const uint2*>(br + row * H + c);
        float2 b0 = unpack_bf16(bb.x), b1 = unpack_bf16(bb.y);
        a.x += b0.x; a.y += b0.y; a.z += b1.x; a.w += b1.y;
      }
      if (br2) {  // the tensor-parallel peer's partial (written over NVLink: L2-only load)
        uint2 bb = __ldcg(reinterpret_cast<const uint2*>(br2 + row * H + c));
        float2 b0 = unpack_bf16(bb.x), b1 = unpack_bf16(bb.y);
        a.x += b0.x; a.y += b0.y; a.z += b1.x; a.w += b1.y;
      }
      v[i] = a;
      ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
      if (out_resid) *reinterpret_cast<float4*>(out_resid + row * H + c) = a;
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  float tot = block_sum(ss, sh);
  float r = rsqrtf(tot / (float)H + eps);
  if (threadIdx.x == 0 && rstd_out) rstd_out[row] = r;
  float s = scale ? *scale : 1.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    int c = (threadIdx.x + i * blockDim.x) * 4;
    if (c < H) {
      float4 ww = *reinterpret_cast<const float4*>(w + c);
      uint2 o;
      o.x = pack_bf16(v[i].x * r * ww.x * s, v[i].y * r * ww.y * s);
      o.y = pack_bf16(v[i].z * r * ww.z * s, v[i].w * r * ww.w * s);
      *reinterpret_cast<uint2*>(y + row * H + c) = o;
    }
  }
  peer_wait_end(pw);
}

// Backward. Block handles ROWS_BWD rows; thread owns VPT float4 column groups.
//   dy_eff = dy * s        (s = *scale if given, else 1)
//   xhat   = x * rstd
//   dx     = rstd * (dy_eff*w - xhat * mean(dy_eff*w*xhat))
//   dresid_out = dresid_in + dx   (dresid_in may alias dresid_out or be null); optional bf16 copy
//   dw    += sum_rows dy_eff * xhat                    (atomic, fp32)
//   dscale+= sum_rows sum_cols dy * xhat * w           (atomic, fp32; only if scale given)
template <int VPT>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const float* __restrict__ x,
                                   const float* __restrict__ rstd, const float* __restrict__ w,
                                   const float* __restrict__ scale, const float* dresid_in, float* dresid_out,
                                   __nv_bfloat16* __restrict__ dresid16, float* __restrict__ dw,
                                   float* __restrict__ dscale, int M, int H, const __nv_bfloat16* dy2,
                                   PeerWait pw) {
  __shared__ float sh[32];
  __shared__ int sh_ok;
  if (!peer_wait_begin(pw, &sh_ok)) {
    peer_wait_end(pw);
    return;
  }
  float4 wv[VPT], dwacc[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    int c = (threadIdx.x + i * blockDim.x) * 4;
    wv[i] = (c < H) ? *reinterpret_cast<const float4*>(w + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    dwacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float s = scale ? *scale : 1.f;
  float ds_acc = 0.f;
  const int r0 = blockIdx.x * ROWS_BWD;
  for (int rr = 0; rr < ROWS_BWD; ++rr) {
    const long long row = r0 + rr;
    if (row >= M) break;
    const float rs = rstd[row];
    float4 g[VPT], xh[VPT];
    float dot = 0.f, dsd = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int c = (threadIdx.x + i * blockDim.x) * 4;
      if (c < H) {
        uint2 bb = *reinterpret_cast<const uint2*>(dy + row * H + c);
        float2 a = unpack_bf16(bb.x), b = unpack_bf16(bb.y);
        if (dy2) {  // the tensor-parallel peer's partial data gradient
          uint2 b2 = __ldcg(reinterpret_cast<const uint2*>(dy2 + row * H + c));
          float2 a2 = unpack_bf16(b2.x), c2 = unpack_bf16(b2.y);
          a.x += a2.x; a.y += a2.y; b.x += c2.x; b.y += c2.y;
        }
        float4 xv = *reinterpret_cast<const float4*>(x + row * H + c);
        xh[i] = make_float4(xv.x * rs, xv.y * rs, xv.z * rs, xv.w * rs);
        g[i] = make_float4(a.x * s, a.y * s, b.x * s, b.y * s);
        dot += g[i].x * wv[i].x * xh[i].x + g[i].y * wv[i].y * xh[i].y + g[i].z * wv[i].z * xh[i].z +
               g[i].w * wv[i].w * xh[i].w;
        if (dscale) dsd += a.x * xh[i].x * wv[i].x + a.y * xh[i].y * wv[i].y + b.x * xh[i].z * wv[i].z + b.y * xh[i].w * wv[i].w;
        dwacc[i].x += g[i].x * xh[i].x; dwacc[i].y += g[i].y * xh[i].y;
        dwacc[i].z += g[i].z * xh[i].z; dwacc[i].w += g[i].w * xh[i].w;
      } else {
        g[i] = xh[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float mean = block_sum(dot, sh) / (float)H;
    ds_acc += dsd;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int c = (threadIdx.x + i * blockDim.x) * 4;
      if (c < H) {
        float4 d = make_float4(rs * (g[i].x * wv[i].x - xh[i].x * mean), rs * (g[i].y * wv[i].y - xh[i].y * mean),
                               rs * (g[i].z * wv[i].z - xh[i].z * mean), rs * (g[i].w * wv[i].w - xh[i].w * mean));
        if (dresid_in) {
          float4 p = *reinterpret_cast<const float4*>(dresid_in + row * H + c);
          d.x += p.x; d.y += p.y; d.z += p.z; d.w += p.w;
        }
        *reinterpret_cast<float4*>(dresid_out + row * H + c) = d;
        if (dresid16) {
          uint2 o;
          o.x = pack_bf16(d.x, d.y);
          o.y = pack_bf16(d.z, d.w);
          *reinterpret_cast<uint2*>(dresid16 + row * H + c) = o;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    int c = (threadIdx.x + i * blockDim.x) * 4;
    if (c < H) atomicAdd(reinterpret_cast<float4*>(dw + c), dwacc[i]);
  }
  if (dscale) {
    float t = block_sum(ds_acc, sh);
    if (threadIdx.x == 0) atomicAdd(dscale, t);
  }
  peer_wait_end(pw);
}

// Warp-per-row backward (H = 128 * VEC): no block-wide barrier per row. All three row loads (dy, x,
// dresid_in) are issued before the row's reduction so each warp keeps ~7.5 KB (H = 768) in flight, and
// w and the per-warp dw partials live in shared memory so two 256-thread blocks fit per SM (<= 128
// registers); the partials are reduced across the block's warps before one atomic per column.
// Blocks per SM: 2 while a row's loads fit 128 registers (VEC <= 8); wider rows keep one block, whose
// 8 warps already hold >= 80 KB in flight.
template <int VEC>
constexpr int rms_bwd_blocks() { return VEC <= 8 ? 2 : 1; }

template <int VEC>
__global__ void __launch_bounds__(256, rms_bwd_blocks<VEC>()) rmsnorm_bwd_warp_kernel(
    const __nv_bfloat16* __restrict__ dy, const float* __restrict__ x, const float* __restrict__ rstd,
    const float* __restrict__ w, const float* __restrict__ scale, const float* dresid_in, float* dresid_out,
    __nv_bfloat16* __restrict__ dresid16, float* __restrict__ dw, float* __restrict__ dscale, int M, int H,
    const __nv_bfloat16* dy2, PeerWait pw) {
  extern __shared__ float red[];  // [8 warps][H] dw partials, then w [H]
  __shared__ int sh_ok;
  if (!peer_wait_begin(pw, &sh_ok)) {
    peer_wait_end(pw);
    return;
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const float s = scale ? *scale : 1.f;
  float* sw = red + 8 * H;
  float* acc = red + wid * H;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4)
    *reinterpret_cast<float4*>(sw + c) = *reinterpret_cast<const float4*>(w + c);
  for (int c = threadIdx.x * 4; c < 8 * H; c += blockDim.x * 4)
    *reinterpret_cast<float4*>(red + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  float ds_acc = 0.f;
  const int gw = blockIdx.x * 8 + wid, nw = gridDim.x * 8;
  for (long long row = gw; row < M; row += nw) {
    const float rs = rstd[row];
    uint2 graw[VEC];
    float4 xh[VEC], pin[VEC];
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 4;
      graw[i] = *reinterpret_cast<const uint2*>(dy + row * H + c);
      if (dy2) {  // the tensor-parallel peer's partial data gradient, summed in fp32 then kept as bf16x2
        const uint2 b2 = __ldcg(reinterpret_cast<const uint2*>(dy2 + row * H + c));
        const float2 a0 = unpack_bf16(graw[i].x), a1 = unpack_bf16(graw[i].y);
        const float2 c0 = unpack_bf16(b2.x), c1 = unpack_bf16(b2.y);
        graw[i].x = pack_bf16(a0.x + c0.x, a0.y + c0.y);
        graw[i].y = pack_bf16(a1.x + c1.x, a1.y + c1.y);
      }
      xh[i] = *reinterpret_cast<const float4*>(x + row * H + c);
      if (dresid_in) pin[i] = *reinterpret_cast<const float4*>(dresid_in + row * H + c);
    }
    float dot = 0.f, dsd = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 4;
      const float4 wv = *reinterpret_cast<const float4*>(sw + c);
      const float2 a = unpack_bf16(graw[i].x), b = unpack_bf16(graw[i].y);
      xh[i] = make_float4(xh[i].x * rs, xh[i].y * rs, xh[i].z * rs, xh[i].w * rs);
      const float4 g = make_float4(a.x * s, a.y * s, b.x * s, b.y * s);
      dot += g.x * wv.x * xh[i].x + g.y * wv.y * xh[i].y + g.z * wv.z * xh[i].z + g.w * wv.w * xh[i].w;
      if (dscale) dsd += a.x * xh[i].x * wv.x + a.y * xh[i].y * wv.y + b.x * xh[i].z * wv.z + b.y * xh[i].w * wv.w;
      float4 av = *reinterpret_cast<float4*>(acc + c);
      av.x += g.x * xh[i].x; av.y += g.y * xh[i].y;
      av.z += g.z * xh[i].z; av.w += g.w * xh[i].w;
      *reinterpret_cast<float4*>(acc + c) = av;
    }
    const float mean = warp_sum(dot) / (float)H;
    ds_acc += dsd;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const int c = (i * 32 + lane) * 4;
      const float4 wv = *reinterpret_cast<const float4*>(sw + c);
      const float2 a = unpack_bf16(graw[i].x), b = unpack_bf16(graw[i].y);
      float4 d = make_float4(rs * (a.x * s * wv.x - xh[i].x * mean), rs * (a.y * s * wv.y - xh[i].y * mean),
                             rs * (b.x * s * wv.z - xh[i].z * mean), rs * (b.y * s * wv.w - xh[i].w * mean));
      if (dresid_in) {
        d.x += pin[i].x; d.y += pin[i].y; d.z += pin[i].z; d.w += pin[i].w;
      }
      *reinterpret_cast<float4*>(dresid_out + row * H + c) = d;
      if (dresid16) {
        uint2 o;
        o.x = pack_bf16(d.x, d.y);
        o.y = pack_bf16(d.z, d.w);
        *reinterpret_cast<uint2*>(dresid16 + row * H + c) = o;
      }
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k * H + c];
    atomicAdd(dw + c, t);
  }
  if (dscale) {
    __shared__ float sh[32];
    float t = block_sum(ds_acc, sh);
    if (threadIdx.x == 0) atomicAdd(dscale, t);
  }
  peer_wait_end(pw);
}

// dE[ids[row]] += g[row]   (fp32, float4 atomics)
__global__ void embedding_bwd_kernel(const float* __restrict__ g, const int* __restrict__ ids, int T, int S,
                                     float* __restrict__ dE, int M, int H) {
  long long row = blockIdx.x;
  long long b = row / T, t = row - b * T;
  const float* src = g + row * H;
  float* dst = dE + (long long)ids[b * S + t] * H;
  for (int c = threadIdx.x * 4; c < H; c += blockDim.x * 4)
    atomicAdd(reinterpret_cast<float4*>(dst + c), *reinterpret_cast<const float4*>(src + c));
}

// Warp-per-row form of the forward (no block barrier, no shared memory): lane l holds float4 chunks
// l, l+32, ..., the row sum of squares is a warp reduction; grid-stride over rows. V = H / 128.
template <int V>
__global__ void __launch_bounds__(256) add_rmsnorm_fwd_warp_kernel(
    const float* __restrict__ x, const __nv_bfloat16* __restrict__ br, const float* __restrict__ emb,
    const int* __restrict__ ids, int T, int S, const float* __restrict__ w, const float* __restrict__ scale,
    float* __restrict__ out_resid, __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, long long M, int H,
    float eps) {
  const int lane = threadIdx.x & 31;
  const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
  const float s = scale ? *scale : 1.f;
  for (long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < M; row += nw) {
    const float* src;
    if (emb) {
      const long long b = row / T, t = row - b * T;
      src = emb + (long long)ids[b * S + t] * H;
    } else {
      src = x + row * H;
    }
    float4 v[V];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = (lane + 32 * i) * 4;
      float4 a = *reinterpret_cast<const float4*>(src + c);
      if (br) {
        const uint2 bb = *reinterpret_cast<const uint2*>(br + row * H + c);
        const float2 b0 = unpack_bf16(bb.x), b1 = unpack_bf16(bb.y);
        a.x += b0.x; a.y += b0.y; a.z += b1.x; a.w += b1.y;
      }
      v[i] = a;
      ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
      if (out_resid) *reinterpret_cast<float4*>(out_resid + row * H + c) = a;
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)H + eps);
    if (lane == 0 && rstd_out) rstd_out[row] = r;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int c = (lane + 32 * i) * 4;
      const float4 ww = *reinterpret_cast<const float4*>(w + c);
      uint2 o;
      o.x = pack_bf16(v[i].x * r * ww.x * s, v[i].y * r * ww.y * s);
      o.y = pack_bf16(v[i].z * r * ww.z * s, v[i].w * r * ww.w * s);
      *reinterpret_cast<uint2*>(y + row * H + c) = o;
    }
  }
}

int threads_for(int H, int vpt) {
  int n = (H / 4 + vpt - 1) / vpt;
  n = ((n + 31) / 32) * 32;
  return n < 32 ? 32 : n;
}

}  // namespace

namespace {

int add_rmsnorm_impl(const float* x, const void* br, const void* br2, const float* emb, const int* ids, int T, int S,
                     const float* w, const float* scale, float* out_resid, void* y, float* rstd, int M, int H, float eps,
                     PeerWait pw, cudaStream_t st) {
  if (H % 4) return -10;
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(br);
  const __nv_bfloat16* b2 = reinterpret_cast<const __nv_bfloat16*>(br2);
  __nv_bfloat16* yy = reinterpret_cast<__nv_bfloat16*>(y);
  if (!b2 && !pw.arrivals && H % 128 == 0 && H <= 2048) {
    long long blocks = ((long long)M + 7) / 8;
    if (blocks > 148 * 8) blocks = 148 * 8;
    switch (H / 128) {
#define DT_RMS_FWD_WARP(V)                                                                                          \
  case V:                                                                                                          \
    add_rmsnorm_fwd_warp_kernel<V><<<(unsigned)blocks, 256, 0, st>>>(x, b, emb, ids, T, S, w, scale, out_resid, yy, \
                                                                     rstd, M, H, eps);                             \
    return (int)cudaGetLastError();
      DT_RMS_FWD_WARP(1) DT_RMS_FWD_WARP(2) DT_RMS_FWD_WARP(3) DT_RMS_FWD_WARP(4)
      DT_RMS_FWD_WARP(5) DT_RMS_FWD_WARP(6) DT_RMS_FWD_WARP(7) DT_RMS_FWD_WARP(8)
      DT_RMS_FWD_WARP(10) DT_RMS_FWD_WARP(12) DT_RMS_FWD_WARP(16)
#undef DT_RMS_FWD_WARP
      default: break;
    }
  }
  if (H <= 4096) {
    int th = threads_for(H, 1);
    add_rmsnorm_fwd_kernel<1><<<M, th, 0, st>>>(x, b, emb, ids, T, S, w, scale, out_resid, yy, rstd, H, eps, b2, pw);
  } else if (H <= 8192) {
    int th = threads_for(H, 2);
    add_rmsnorm_fwd_kernel<2><<<M, th, 0, st>>>(x, b, emb, ids, T, S, w, scale, out_resid, yy, rstd, H, eps, b2, pw);
  } else {
    return -11;
  }
  return (int)cudaGetLastError();
}

int rmsnorm_bwd_impl(const void* dy, const void* dy2, const float* x, const float* rstd, const float* w,
                     const float* scale, const float* dresid_in, float* dresid_out, void* dresid16, float* dw,
                     float* dscale, int M, int H, PeerWait pw, cudaStream_t st) {
  if (H % 4) return -10;
  int blocks = (M + ROWS_BWD - 1) / ROWS_BWD;
  const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(dy);
  const __nv_bfloat16* d2 = reinterpret_cast<const __nv_bfloat16*>(dy2);
  auto d16 = reinterpret_cast<__nv_bfloat16*>(dresid16);
  if (H % 128 == 0 && H <= 2048) {
    int wb = (M + 7) / 8;
    const int per_sm = (H / 128) <= 8 ? 2 : 1;
    if (wb > 148 * per_sm) wb = 148 * per_sm;
    size_t sm = sizeof(float) * 9 * H;
#define DT_RMS_WARP(V)                                                                                       \
  case V:                                                                                                   \
    if (sm > 48 * 1024) cudaFuncSetAttribute(rmsnorm_bwd_warp_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm); \
    rmsnorm_bwd_warp_kernel<V><<<wb, 256, sm, st>>>(d, x, rstd, w, scale, dresid_in, dresid_out, d16, dw, dscale, M, H, \
                                                    d2, pw);                                                 \
    return (int)cudaGetLastError();
    switch (H / 128) {
      DT_RMS_WARP(1) DT_RMS_WARP(2) DT_RMS_WARP(3) DT_RMS_WARP(4) DT_RMS_WARP(5) DT_RMS_WARP(6) DT_RMS_WARP(8)
      DT_RMS_WARP(10) DT_RMS_WARP(12) DT_RMS_WARP(16)
      default: break;
    }
#undef DT_RMS_WARP
  }
  if (H <= 4096) {
    rmsnorm_bwd_kernel<1><<<blocks, threads_for(H, 1), 0, st>>>(d, x, rstd, w, scale, dresid_in, dresid_out, d16, dw,
                                                                dscale, M, H, d2, pw);
  } else if (H <= 8192) {
    rmsnorm_bwd_kernel<2><<<blocks, threads_for(H, 2), 0, st>>>(d, x, rstd, w, scale, dresid_in, dresid_out, d16, dw,
                                                                dscale, M, H, d2, pw);
  } else {
    return -11;
  }
  return (int)cudaGetLastError();
}

}  // namespace

// resid_out = (emb ? emb[ids] : x) + br ;  y = bf16(rmsnorm(resid_out) * w * scale)
DT_API int dt_add_rmsnorm_fwd(const float* x, const void* br, const float* emb, const int* ids, int T, int S,
                              const float* w, const float* scale, float* out_resid, void* y, float* rstd, int M,
                              int H, float eps, cudaStream_t st) {
  return add_rmsnorm_impl(x, br, nullptr, emb, ids, T, S, w, scale, out_resid, y, rstd, M, H, eps, PeerWait{}, st);
}

// Tensor-parallel form: resid_out = x + br + br2 with br2 the peer's partial in this GPU's receive buffer,
// waited for through the arrival / consumed counters (PeerWait).
DT_API int dt_add_rmsnorm_fwd_tp(const float* x, const void* br, const void* br2, const float* w, const float* scale,
                                 float* out_resid, void* y, float* rstd, int M, int H, float eps,
                                 const unsigned* arrivals, unsigned* consumed, unsigned* done_blocks,
                                 cudaStream_t st) {
  return add_rmsnorm_impl(x, br, br2, nullptr, nullptr, 1, 1, w, scale, out_resid, y, rstd, M, H, eps,
                          PeerWait{arrivals, consumed, done_blocks}, st);
}

DT_API int dt_rmsnorm_bwd(const void* dy, const float* x, const float* rstd, const float* w, const float* scale,
                          const float* dresid_in, float* dresid_out, void* dresid16, float* dw, float* dscale, int M,
                          int H, cudaStream_t st) {
  return rmsnorm_bwd_impl(dy, nullptr, x, rstd, w, scale, dresid_in, dresid_out, dresid16, dw, dscale, M, H,
                          PeerWait{}, st);
}

// Tensor-parallel form: dy + dy2 with dy2 the peer's partial data gradient in the receive buffer.
DT_API int dt_rmsnorm_bwd_tp(const void* dy, const void* dy2, const float* x, const float* rstd, const float* w,
                             const float* scale, const float* dresid_in, float* dresid_out, void* dresid16, float* dw,
                             float* dscale, int M, int H, const unsigned* arrivals, unsigned* consumed,
                             unsigned* done_blocks, cudaStream_t st) {
  return rmsnorm_bwd_impl(dy, dy2, x, rstd, w, scale, dresid_in, dresid_out, dresid16, dw, dscale, M, H,
                          PeerWait{arrivals, consumed, done_blocks}, st);
}

DT_API int dt_embedding_bwd(const float* g, const int* ids, int T, int S, float* dE, int M, int H, cudaStream_t st) {
  if (H % 4) return -10;
  int th = H / 4 < 256 ? ((H / 4 + 31) / 32) * 32 : 256;
  embedding_bwd_kernel<<<M, th, 0, st>>>(g, ids, T, S, dE, M, H);
  return (int)cudaGetLastError();
}
