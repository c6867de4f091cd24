// Causal GQA flash attention, forward and backward, bf16 in / fp32 softmax statistics.
// LSE and delta rows are [B, nh, Tp] with Tp = T rounded up to a multiple of 4 (16-byte aligned rows).
//
// Reads q/k/v straight out of the fused QKV activation ([B*T, (nh+2nkv)*D], after bias+RoPE): query
// head h uses kv head h / (nh/nkv) (reference expand_kv_heads, core/model/src/model.rs:127-138, by
// indexing instead of materialising). Scores are scaled by 1/sqrt(D) and causally masked
// (model.rs:246-256); the reference's additive -1e4 mask and this kernel's exact masking agree to far
// below bf16 resolution. No S x S matrix is ever stored: the forward keeps the online-softmax
// statistics per row and saves LSE for the backward.
//
// Tensor-core path: warp-level mma.sync m16n8k16 (bf16 -> fp32) with ldmatrix-fed fragments and
// cp.async double-buffered K/V tiles in XOR-swizzled shared memory.
//   forward : CTA = (64 queries of one head), 4 warps x 16 rows, K/V tiles of 64 keys.
//   backward: CTA = (64 keys of one kv head), 4 warps x 16 keys; loops over the kv group's query
//             heads and the causal query blocks, accumulating dK/dV in registers (no atomics) and
//             adding dQ with fp32 atomics into a caller-provided accumulator.
#include "common.cuh"

namespace {

constexpr int BM = 64;   // queries per forward CTA
constexpr int BN = 64;   // keys per tile
constexpr int NT = 128;  // threads (4 warps)
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

__device__ __forceinline__ int swz(int row, int col, int D) {
  // element offset in a [rows][D] bf16 tile with 16-byte chunks XOR-swizzled by the row (kept inside
  // the row's D/8 chunks), so the 8 row addresses of one ldmatrix hit distinct bank groups
  const int mask = (D >= 64 ? 8 : D / 8) - 1;
  int chunk = col >> 3;
  return row * D + ((chunk ^ (row & mask)) << 3) + (col & 7);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  unsigned s = smem_u32(smem);
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Load a [64][D] tile whose row r lives at base + (row0 + r) * ld (rows >= rows_valid zero-filled).
template <int D>
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, const __nv_bfloat16* base, long long ld, int row0,
                                          int rows_valid) {
  constexpr int CH = D / 8;
  for (int i = threadIdx.x; i < 64 * CH; i += NT) {
    int r = i / CH, c = i % CH;
    bool ok = (row0 + r) < rows_valid;
    const __nv_bfloat16* g = base + (long long)(ok ? row0 + r : 0) * ld + c * 8;
    cp_async16(s + swz(r, c * 8, D), g, ok);
  }
}

// Warp computes acc[16 x 64] = A(16 rows of `sa`, starting at arow) . B^T where B rows are the 64 rows of `sb`.
template <int D>
__device__ __forceinline__ void mm_rows_x_rowsT(float (&acc)[8][4], const __nv_bfloat16* sa, int arow,
                                                const __nv_bfloat16* sb) {
  const int lane = threadIdx.x & 31;
  const int j = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    uint32_t a[4];
    ldsm_x4(a, sa + swz(arow + (j & 1) * 8 + rr, kk * 16 + (j >> 1) * 8, D));
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      uint32_t b[4];
      ldsm_x4(b, sb + swz(np * 16 + (j >> 1) * 8 + rr, kk * 16 + (j & 1) * 8, D));
      mma16816(acc[2 * np], a, b[0], b[1]);
      mma16816(acc[2 * np + 1], a, b[2], b[3]);
    }
  }
}

// Warp: out[16 x D] += P[16 x 64] (register A fragments from an 8x4 accumulator layout) . Vtile[64 x D]
template <int D>
__device__ __forceinline__ void mm_p_x_tile(float (&out)[D / 8][4], const float (&p)[8][4], const __nv_bfloat16* sv) {
  const int lane = threadIdx.x & 31;
  const int j = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4];
    a[0] = pack_bf16(p[2 * kk][0], p[2 * kk][1]);
    a[1] = pack_bf16(p[2 * kk][2], p[2 * kk][3]);
    a[2] = pack_bf16(p[2 * kk + 1][0], p[2 * kk + 1][1]);
    a[3] = pack_bf16(p[2 * kk + 1][2], p[2 * kk + 1][3]);
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t b[4];
      ldsm_x4_t(b, sv + swz(kk * 16 + (j & 1) * 8 + rr, dp * 16 + (j >> 1) * 8, D));
      mma16816(out[2 * dp], a, b[0], b[1]);
      mma16816(out[2 * dp + 1], a, b[2], b[3]);
    }
  }
}

// ─────────────────────────────── forward ───────────────────────────────
template <int D>
__global__ void __launch_bounds__(NT) attn_fwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                      __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                                                      int B, int T, int nh, int nkv, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sk = sq + 64 * D;   // [2][64*D]
  __nv_bfloat16* sv = sk + 2 * 64 * D;

  const int nqb = (T + BM - 1) / BM;
  // heavy (late) query blocks first
  const int qb = nqb - 1 - (blockIdx.x % nqb);
  const int bh = blockIdx.x / nqb;
  const int h = bh % nh, b = bh / nh;
  const int g = h / (nh / nkv);
  const long long W = (long long)(nh + 2 * nkv) * D;
  const __nv_bfloat16* qbase = qkv + (long long)b * T * W + h * D;
  const __nv_bfloat16* kbase = qkv + (long long)b * T * W + (nh + g) * D;
  const __nv_bfloat16* vbase = qkv + (long long)b * T * W + (nh + nkv + g) * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;

  load_tile<D>(sq, qbase, W, qb * BM, T);
  load_tile<D>(sk, kbase, W, 0, T);
  load_tile<D>(sv, vbase, W, 0, T);
  cp_async_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_[2] = {-INFINITY, -INFINITY}, l_[2] = {0.f, 0.f};
  const float sl2 = scale * LOG2E;
  const int q0 = qb * BM + warp * 16 + gid;  // rows q0 and q0 + 8
  const int nkb = qb + 1;                     // causal: key blocks 0..qb

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) {
      load_tile<D>(sk + (buf ^ 1) * 64 * D, kbase, W, (kb + 1) * BN, T);
      load_tile<D>(sv + (buf ^ 1) * 64 * D, vbase, W, (kb + 1) * BN, T);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float s[8][4];
    mm_rows_x_rowsT<D>(s, sq, warp * 16, sk + buf * 64 * D);
    const bool diag = (kb == qb);
    const int kbase_idx = kb * BN;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int key = kbase_idx + n * 8 + tig * 2 + (e & 1);
        int q = q0 + (e >> 1) * 8;
        float v = s[n][e] * sl2;
        if ((diag && key > q) || key >= T) v = -INFINITY;
        s[n][e] = v;
      }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * i], s[n][2 * i + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float mnew = fmaxf(m_[i], mx);
      float msafe = (mnew == -INFINITY) ? 0.f : mnew;
      float alpha = exp2f(m_[i] - msafe);
      float rs = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        float p0 = exp2f(s[n][2 * i] - msafe), p1 = exp2f(s[n][2 * i + 1] - msafe);
        s[n][2 * i] = p0;
        s[n][2 * i + 1] = p1;
        rs += p0 + p1;
      }
      l_[i] = l_[i] * alpha + rs;
      m_[i] = mnew;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][2 * i] *= alpha;
        o[dt][2 * i + 1] *= alpha;
      }
    }
    mm_p_x_tile<D>(o, s, sv + buf * 64 * D);
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float l = l_[i];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const int q = q0 + i * 8;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    if (q < T) {
      __nv_bfloat16* orow = out + ((long long)b * T + q) * ((long long)nh * D) + h * D;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        *reinterpret_cast<uint32_t*>(orow + dt * 8 + tig * 2) = pack_bf16(o[dt][2 * i] * inv, o[dt][2 * i + 1] * inv);
      }
      if (tig == 0) lse[((long long)b * nh + h) * ((T + 3) & ~3) + q] = (m_[i] + log2f(l)) * LN2;
    }
  }
}

// ─────────────────────────────── backward ───────────────────────────────
// delta[b,h,q] = sum_d dO * O. Thread = 8 consecutive elements of one row (16-byte loads, a warp reads 512
// contiguous bytes of each operand); the D/8 threads of one (row, head) sit in consecutive lanes and sum
// by shuffles, the first writes delta.
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ dout,
                                    float* __restrict__ delta, int B, int T, int nh, int D) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;  // 8-element chunk
  const int cpr = nh * D / 8;                                             // chunks per row
  const long long total = (long long)B * T * cpr;
  float acc = 0.f;
  if (i < total) {
    const uint4 a = reinterpret_cast<const uint4*>(out)[i], e = reinterpret_cast<const uint4*>(dout)[i];
    const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, ee[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = unpack_bf16(aa[k]), y = unpack_bf16(ee[k]);
      acc += x.x * y.x + x.y * y.y;
    }
  }
  const int g = D / 8;  // lanes per (row, head): divides 32, so a group never straddles warps
  for (int o = g >> 1; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (i < total && (threadIdx.x & (g - 1)) == 0) {
    const long long row = i / cpr;
    const int h = (int)((i - row * cpr) / g);
    const long long b = row / T, t = row - b * T;
    delta[(b * nh + h) * ((T + 3) & ~3) + t] = acc;
  }
}

template <int D>
__global__ void __launch_bounds__(NT) attn_bwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                      const __nv_bfloat16* __restrict__ dout,
                                                      const float* __restrict__ lse, const float* __restrict__ delta,
                                                      __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dq_acc,
                                                      int B, int T, int nh, int nkv, float scale) {
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sv = sk + 64 * D;
  __nv_bfloat16* sq = sv + 64 * D;
  __nv_bfloat16* sdo = sq + 64 * D;
  __nv_bfloat16* sds = sdo + 64 * D;  // [64 keys][64 q]
  float* slse = reinterpret_cast<float*>(sds + 64 * 64);
  float* sdel = slse + 64;

  const int nkb = (T + BN - 1) / BN;
  const int kb = blockIdx.x % nkb;  // light (late) key blocks last: reverse order below
  const int kbr = kb;
  const int bg = blockIdx.x / nkb;
  const int g = bg % nkv, b = bg / nkv;
  const int G = nh / nkv;
  const long long W = (long long)(nh + 2 * nkv) * D;
  const long long HD = (long long)nh * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int j = lane >> 3, rr = lane & 7;
  const __nv_bfloat16* kbase = qkv + (long long)b * T * W + (nh + g) * D;
  const __nv_bfloat16* vbase = qkv + (long long)b * T * W + (nh + nkv + g) * D;

  load_tile<D>(sk, kbase, W, kbr * BN, T);
  load_tile<D>(sv, vbase, W, kbr * BN, T);
  cp_async_commit();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  const float sl2 = scale * LOG2E;
  const int key0 = kbr * BN + warp * 16 + gid;  // rows key0, key0 + 8
  const int nqb = (T + BM - 1) / BM;

  for (int hh = 0; hh < G; ++hh) {
    const int h = g * G + hh;
    const __nv_bfloat16* qbase = qkv + (long long)b * T * W + h * D;
    const __nv_bfloat16* dobase = dout + (long long)b * T * HD + h * D;
    for (int qb = kbr; qb < nqb; ++qb) {
      __syncthreads();  // previous iteration done with sq/sdo/sds
      load_tile<D>(sq, qbase, W, qb * BM, T);
      load_tile<D>(sdo, dobase, HD, qb * BM, T);
      cp_async_commit();
      if (threadIdx.x < 64) {
        int q = qb * BM + threadIdx.x;
        long long idx = ((long long)b * nh + h) * ((T + 3) & ~3) + q;
        slse[threadIdx.x] = (q < T) ? lse[idx] * LOG2E : INFINITY;
        sdel[threadIdx.x] = (q < T) ? delta[idx] : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();
      // S^T = K Q^T  (16 keys x 64 queries per warp)
      float st[8][4];
      mm_rows_x_rowsT<D>(st, sk, warp * 16, sq);
      // dP^T = V dO^T
      float dpt[8][4];
      mm_rows_x_rowsT<D>(dpt, sv, warp * 16, sdo);
      const bool diag = (qb == kbr);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int ql = n * 8 + tig * 2 + (e & 1);
          int q = qb * BM + ql;
          int key = key0 + (e >> 1) * 8;
          float p = exp2f(st[n][e] * sl2 - slse[ql]);
          if ((diag && q < key) || q >= T || key >= T) p = 0.f;
          st[n][e] = p;                              // P^T
          dpt[n][e] = p * (dpt[n][e] - sdel[ql]);    // dS^T (unscaled)
        }
      }
      // dV += P^T dO ; dK += dS^T Q
      mm_p_x_tile<D>(dv, st, sdo);
      mm_p_x_tile<D>(dk, dpt, sq);
      // stash dS^T for the dQ product
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        int col = n * 8 + tig * 2;
        int r0 = warp * 16 + gid;
        *reinterpret_cast<uint32_t*>(sds + swz(r0, col, 64)) = pack_bf16(dpt[n][0], dpt[n][1]);
        *reinterpret_cast<uint32_t*>(sds + swz(r0 + 8, col, 64)) = pack_bf16(dpt[n][2], dpt[n][3]);
      }
      __syncthreads();
      // dQ[16 q of this warp x D] = dS[q, keys] . K[keys, D]
      float dq[D / 8][4];
#pragma unroll
      for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        // A[q][key] from dS^T stored [key][q]: transposed ldmatrix
        ldsm_x4_t(a, sds + swz(kk * 16 + (j >> 1) * 8 + rr, warp * 16 + (j & 1) * 8, 64));
#pragma unroll
        for (int dp = 0; dp < D / 16; ++dp) {
          uint32_t bb[4];
          ldsm_x4_t(bb, sk + swz(kk * 16 + (j & 1) * 8 + rr, dp * 16 + (j >> 1) * 8, D));
          mma16816(dq[2 * dp], a, bb[0], bb[1]);
          mma16816(dq[2 * dp + 1], a, bb[2], bb[3]);
        }
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        int q = qb * BM + warp * 16 + gid + i * 8;
        if (q < T) {
          float* dst = dq_acc + ((long long)b * T + q) * HD + h * D;
#pragma unroll
          for (int dt = 0; dt < D / 8; ++dt) {
            atomicAdd(reinterpret_cast<float2*>(dst + dt * 8 + tig * 2),
                      make_float2(dq[dt][2 * i] * scale, dq[dt][2 * i + 1] * scale));
          }
        }
      }
    }
  }
  // write dK (scaled) and dV for this key block
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    int key = key0 + i * 8;
    if (key < T) {
      __nv_bfloat16* krow = dqkv + ((long long)b * T + key) * W + (nh + g) * D;
      __nv_bfloat16* vrow = dqkv + ((long long)b * T + key) * W + (nh + nkv + g) * D;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        *reinterpret_cast<uint32_t*>(krow + dt * 8 + tig * 2) = pack_bf16(dk[dt][2 * i] * scale, dk[dt][2 * i + 1] * scale);
        *reinterpret_cast<uint32_t*>(vrow + dt * 8 + tig * 2) = pack_bf16(dv[dt][2 * i], dv[dt][2 * i + 1]);
      }
    }
  }
}

// dqkv[:, q heads] = bf16(dq_acc)
__global__ void dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, long long M,
                                  int HD, long long W) {
  long long n = M * (HD / 4);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long row = i / (HD / 4);
    int c = (int)(i - row * (HD / 4)) * 4;
    float4 v = *reinterpret_cast<const float4*>(dq_acc + row * HD + c);
    uint2 o;
    o.x = pack_bf16(v.x, v.y);
    o.y = pack_bf16(v.z, v.w);
    *reinterpret_cast<uint2*>(dqkv + row * W + c) = o;
  }
}

template <int D>
int fwd_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int B, int T, int nh, int nkv, float scale,
               cudaStream_t st) {
  size_t smem = (size_t)(64 * D + 4 * 64 * D) * 2;
  static bool set = false;
  if (!set) {
    DT_CUDA_RET(cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    set = true;
  }
  int nqb = (T + BM - 1) / BM;
  attn_fwd_kernel<D><<<B * nh * nqb, NT, smem, st>>>(qkv, out, lse, B, T, nh, nkv, scale);
  return (int)cudaGetLastError();
}

template <int D>
int bwd_launch(const __nv_bfloat16* qkv, const __nv_bfloat16* dout, const float* lse, const float* delta,
               __nv_bfloat16* dqkv, float* dq_acc, int B, int T, int nh, int nkv, float scale, cudaStream_t st) {
  size_t smem = (size_t)(4 * 64 * D + 64 * 64) * 2 + 2 * 64 * 4;
  static bool set = false;
  if (!set) {
    DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    set = true;
  }
  int nkb = (T + BN - 1) / BN;
  attn_bwd_kernel<D><<<B * nkv * nkb, NT, smem, st>>>(qkv, dout, lse, delta, dqkv, dq_acc, B, T, nh, nkv, scale);
  return (int)cudaGetLastError();
}

}  // namespace

DT_API int dt_attn_fwd(const void* qkv, void* out, float* lse, int B, int T, int nh, int nkv, int D, float scale,
                       cudaStream_t st) {
  if (nh % nkv) return -10;
  auto q = reinterpret_cast<const __nv_bfloat16*>(qkv);
  auto o = reinterpret_cast<__nv_bfloat16*>(out);
  if (D == 64) return fwd_launch<64>(q, o, lse, B, T, nh, nkv, scale, st);
  if (D == 128) return fwd_launch<128>(q, o, lse, B, T, nh, nkv, scale, st);
  if (D == 16) return fwd_launch<16>(q, o, lse, B, T, nh, nkv, scale, st);
  if (D == 32) return fwd_launch<32>(q, o, lse, B, T, nh, nkv, scale, st);
  return -11;
}

DT_API int dt_attn_bwd(const void* qkv, const void* out, const void* dout, const float* lse, void* dqkv,
                       float* dq_acc, float* delta, int B, int T, int nh, int nkv, int D, float scale,
                       cudaStream_t st) {
  if (nh % nkv) return -10;
  auto q = reinterpret_cast<const __nv_bfloat16*>(qkv);
  auto o = reinterpret_cast<const __nv_bfloat16*>(out);
  auto d = reinterpret_cast<const __nv_bfloat16*>(dout);
  auto dq = reinterpret_cast<__nv_bfloat16*>(dqkv);
  long long M = (long long)B * T;
  DT_CUDA_RET(cudaMemsetAsync(dq_acc, 0, sizeof(float) * M * nh * D, st));
  long long items = M * nh * (D / 8);
  attn_bwd_pre_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(o, d, delta, B, T, nh, D);
  int rc;
  if (D == 64) rc = bwd_launch<64>(q, d, lse, delta, dq, dq_acc, B, T, nh, nkv, scale, st);
  else if (D == 128) rc = bwd_launch<128>(q, d, lse, delta, dq, dq_acc, B, T, nh, nkv, scale, st);
  else if (D == 16) rc = bwd_launch<16>(q, d, lse, delta, dq, dq_acc, B, T, nh, nkv, scale, st);
  else if (D == 32) rc = bwd_launch<32>(q, d, lse, delta, dq, dq_acc, B, T, nh, nkv, scale, st);
  else return -11;
  if (rc) return rc;
  long long n = M * (nh * D / 4);
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  dq_convert_kernel<<<(unsigned)blocks, 256, 0, st>>>(dq_acc, dq, M, nh * D, (long long)(nh + 2 * nkv) * D);
  return (int)cudaGetLastError();
}

// delta = rowsum(dO * O) per (row, head) into [B, nh, Tp] (the tcgen05 backward's pre-pass).
DT_API int dt_attn_bwd_delta(const void* out, const void* dout, float* delta, int B, int T, int nh, int D,
                             cudaStream_t st) {
  if (D % 8 || 32 % (D / 8)) return -10;
  long long items = (long long)B * T * nh * (D / 8);
  attn_bwd_pre_kernel<<<(unsigned)((items + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(out), reinterpret_cast<const __nv_bfloat16*>(dout), delta, B, T, nh, D);
  return (int)cudaGetLastError();
}
