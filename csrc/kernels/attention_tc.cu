// Causal GQA flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM), d = 64 / 128.
//
// Same contract as the mma.sync kernels in attention.cu (q/k/v read from the fused QKV activation,
// query head h uses kv head h / (nh/nkv), out [B*T, nh*D] bf16, lse [B, nh, T] fp32 natural log).
//
// One CTA = 128 query rows of one (batch, head); 6 warps:
//   warp 0     TMA producer: Q once, then K/V tiles of 128 keys into a 2-stage ring (3-D tensor map
//              [B, T, W] so rows past T are zero-filled per sequence; no cluster multicast)
//   warp 1     single-thread tcgen05.mma issuer: S = Q K^T (M=128, N=128) into TMEM, then
//              O += P V (M=128, N=D, K=128) with P from shared memory and V as an MN-major operand
//   warps 2-5  softmax: thread i owns query row i = TMEM lane i. Two passes over S (max, then
//              exp2 / row-sum / bf16 P written in the 128-byte-swizzled K-major layout the MMA reads).
//              The running max is only raised when it grows by more than 8 (log2 units); O in TMEM is
//              rescaled (tcgen05.ld/st) only then, otherwise P is taken against the stale max (values
//              stay <= 2^8, exact after normalisation).
// TMEM: S at columns [0,128), O at [128, 128+D) -> 256 columns, so two CTAs share an SM (d = 64) and
// one CTA's softmax overlaps the other's MMAs. Every mbarrier wait is bounded.
#include "common.cuh"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

namespace {

constexpr int BQ = 128, BKV = 128, NTH = 192;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float LN2_F = 0.6931471805599453f;
constexpr float RESCALE_THRESHOLD = 8.0f;

template <int D>
struct FCfg {
  static constexpr int QB = BQ * D * 2;        // Q tile bytes
  static constexpr int KB = BKV * D * 2;       // K tile bytes
  static constexpr int VB = BKV * D * 2;       // V tile bytes
  static constexpr int PB = BQ * BKV * 2;      // P tile bytes
  static constexpr int STAGES = 2;
  // no alignment slack: with no static shared memory the dynamic window starts 1024-aligned
  // (checked at run time), which keeps two d=64 CTAs within one SM's 228 KB
  static constexpr int SMEM = QB + STAGES * (KB + VB) + PB + 256;
  static constexpr int TMEM_COLS = 256;
};

template <int D>
__global__ void __launch_bounds__(NTH, 1) attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV,
                                                              __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                                                              int B, int T, int nh, int nkv, float scale) {
  using C = FCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // uniform across the CTA; nothing allocated yet
    if (threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 499);
    return;
  }
  uint8_t* sm = smem_raw;
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + C::QB;                 // [STAGES][KB]
  uint8_t* sV = sK + C::STAGES * C::KB;     // [STAGES][VB]
  uint8_t* sP = sV + C::STAGES * C::VB;     // [PB]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sP + C::PB);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;   // [2]
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* s_full = bar + 5;
  uint64_t* s_free = bar + 6;
  uint64_t* p_full = bar + 7;
  uint64_t* pv_done = bar + 8;
  uint64_t* drain = bar + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (T + BQ - 1) / BQ;
  const int qb = nqb - 1 - (blockIdx.x % nqb);  // heavy (long) query blocks first
  const int bh = blockIdx.x / nqb;
  const int h = bh % nh, b = bh / nh;
  const int g = h / (nh / nkv);
  const int nkb = qb + 1;  // causal: key blocks 0..qb (BKV == BQ)

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      const int xq = h * D, xk = (nh + g) * D, xv = (nh + nkv + g) * D;
      mbar_arrive_expect_tx(q_full, C::QB);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_3d(sQ + c * (BQ * 128), &tmQKV, q_full, xq + 64 * c, qb * BQ, b);
      for (int j = 0; j < nkb; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait_bounded(&kv_empty[st], ((j >> 1) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 400, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], C::KB + C::VB);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sK + st * C::KB + c * (BKV * 128), &tmQKV, &kv_full[st], xk + 64 * c, j * BKV, b);
          tma_load_3d(sV + st * C::VB + c * (BKV * 128), &tmQKV, &kv_full[st], xv + 64 * c, j * BKV, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(BQ, BKV, 0, 0);
      constexpr uint32_t idO = umma_idesc_bf16(BQ, D, 0, 1);
      bool ok = mbar_wait_bounded(q_full, 0, DT_ERR_TIMEOUT_FULL, 410, abort_flag);
      const uint32_t aq = smem_u32(sQ);
      bool issued = false;
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait_bounded(p_full, jj & 1, DT_ERR_TIMEOUT_FULL, 413, abort_flag)) return false;
        tc_fence_after();
        const uint32_t ap = smem_u32(sP), bv = smem_u32(sV + (jj & 1) * C::VB);
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k) {
          uint64_t ad = umma_smem_desc_sw128(ap + (k >> 2) * (BQ * 128) + (k & 3) * 32, 16, 1024);
          uint64_t bd = umma_smem_desc_sw128(bv + k * 2048, BKV * 128, 1024);
          umma_bf16(tO, ad, bd, idO, (jj > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(pv_done);
        umma_commit(&kv_empty[jj & 1]);
        return true;
      };
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait_bounded(&kv_full[st], (j >> 1) & 1, DT_ERR_TIMEOUT_FULL, 411, abort_flag)) { ok = false; break; }
        if (j > 0 && !mbar_wait_bounded(s_free, (j - 1) & 1, DT_ERR_TIMEOUT_TMEM, 412, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t bk = smem_u32(sK + st * C::KB);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          uint64_t ad = umma_smem_desc_sw128(aq + (k >> 2) * (BQ * 128) + (k & 3) * 32, 16, 1024);
          uint64_t bd = umma_smem_desc_sw128(bk + (k >> 2) * (BKV * 128) + (k & 3) * 32, 16, 1024);
          umma_bf16(tS, ad, bd, idS, k > 0 ? 1u : 0u);
        }
        issued = true;
        umma_commit(s_full);
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(nkb - 1);
      if (!ok && issued) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    // ───────────── softmax warps: row r = TMEM lane r ─────────────
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int q = qb * BQ + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = scale * LOG2E_F;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // one lane waits, the warp follows: keeps every lane on the same path around warp-collective TMEM ops
    auto wwait = [&](uint64_t* bb, uint32_t par, int site) -> bool {
      int okl = 1;
      if (lane == 0) okl = mbar_wait_bounded(bb, par, DT_ERR_TIMEOUT_TMEM, site, abort_flag) ? 1 : 0;
      okl = __shfl_sync(0xffffffffu, okl, 0);
      __syncwarp();
      return okl != 0;
    };
    for (int j = 0; j < nkb; ++j) {
      if (!wwait(s_full, j & 1, 420)) { ok = false; break; }
      tc_fence_after();
      const int key0 = j * BKV;
      const bool diag = (j == qb);
      // pass A: row max over the 128 scores (masked)
      float mx = -INFINITY;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(tS + lane_off + h2 * 64, v[0]);
        tmem_ld_32x32b_x32(tS + lane_off + h2 * 64 + 32, v[1]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int key = key0 + h2 * 64 + c;
          float sv = __uint_as_float(v[c >> 5][c & 31]) * sl2;
          if ((diag && key > q) || key >= T) sv = -INFINITY;
          mx = fmaxf(mx, sv);
        }
      }
      // stale-max policy: raise the reference max only when it grows by more than the threshold
      float m_use = m_run;
      bool resc = false;
      if (mx > m_run + RESCALE_THRESHOLD || m_run == -INFINITY) {
        m_use = mx;
        resc = (m_run != -INFINITY);
      }
      const float m_safe = (m_use == -INFINITY) ? 0.f : m_use;
      const float alpha = resc ? ex2_approx(m_run - m_use) : 1.f;
      // P buffer and O are busy until the previous P.V has completed
      if (j > 0 && !wwait(pv_done, (j - 1) & 1, 421)) { ok = false; break; }
      tc_fence_after();
      // pass B: p = exp2(s - m), row sum, bf16 P tile in the swizzled K-major layout
      float rs = 0.f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(tS + lane_off + h2 * 64, v[0]);
        tmem_ld_32x32b_x32(tS + lane_off + h2 * 64 + 32, v[1]);
        tmem_ld_wait();
        if (h2 == 1) {
          tc_fence_before();
          mbar_arrive(s_free);  // S fully in registers: the next Q K^T may overwrite it
        }
        uint8_t* prow = sP + h2 * (BQ * 128) + r * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          float pv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int c = ch * 8 + e;
            const int key = key0 + h2 * 64 + c;
            float sv = __uint_as_float(v[c >> 5][c & 31]) * sl2;
            float p = ((diag && key > q) || key >= T) ? 0.f : ex2_approx(sv - m_safe);
            pv[e] = p;
            rs += p;
          }
          uint4 w;
          w.x = pack_bf16(pv[0], pv[1]);
          w.y = pack_bf16(pv[2], pv[3]);
          w.z = pack_bf16(pv[4], pv[5]);
          w.w = pack_bf16(pv[6], pv[7]);
          *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) * 16)) = w;
        }
      }
      l_run = l_run * alpha + rs;
      m_run = m_use;
      // rescale O (warp-collective TMEM access; lanes that need no rescale multiply by 1)
      if (__any_sync(0xffffffffu, resc) && j > 0) {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + lane_off + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + lane_off + c0, o);
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // epilogue: O / l -> bf16 rows of `out`, lse
    if (ok && wwait(pv_done, (nkb - 1) & 1, 422)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = out + ((long long)b * T + q) * ((long long)nh * D) + h * D;
#pragma unroll
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tO + lane_off + c0, o);
        tmem_ld_wait();
        if (q < T) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = pack_bf16(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = pack_bf16(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = pack_bf16(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c0 + 8 * v) = w;
          }
        }
      }
      if (q < T) lse[((long long)b * nh + h) * ((T + 3) & ~3) + q] = (m_run + log2f(l_run)) * LN2_F;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;
std::once_flag g_enc_once;

int qkv_map(CUtensorMap* m, const void* qkv, int B, int T, long long W) {
  std::call_once(g_enc_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_enc) return -2;
  cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)T, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(W * 2), (cuuint64_t)(W * 2 * T)};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(qkv), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

template <int D>
int fwd_tc_launch(const void* qkv, void* out, float* lse, int B, int T, int nh, int nkv, float scale, cudaStream_t st) {
  using C = FCfg<D>;
  long long W = (long long)(nh + 2 * nkv) * D;
  if ((W * 2) % 16 || (reinterpret_cast<uintptr_t>(qkv) & 15)) return -10;
  CUtensorMap m;
  int rc = qkv_map(&m, qkv, B, T, W);
  if (rc) return rc;
  static bool set = false;
  if (!set) {
    DT_CUDA_RET(cudaFuncSetAttribute(attn_fwd_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    set = true;
  }
  int nqb = (T + BQ - 1) / BQ;
  attn_fwd_tc_kernel<D><<<B * nh * nqb, NTH, C::SMEM, st>>>(m, reinterpret_cast<__nv_bfloat16*>(out), lse, B, T, nh,
                                                             nkv, scale);
  return (int)cudaGetLastError();
}

}  // namespace

// tcgen05 forward; D must be 64 or 128 (other head dims use dt_attn_fwd).
DT_API int dt_attn_fwd_tc(const void* qkv, void* out, float* lse, int B, int T, int nh, int nkv, int D, float scale,
                          cudaStream_t st) {
  if (nh % nkv) return -10;
  if (D == 64) return fwd_tc_launch<64>(qkv, out, lse, B, T, nh, nkv, scale, st);
  if (D == 128) return fwd_tc_launch<128>(qkv, out, lse, B, T, nh, nkv, scale, st);
  return -11;
}

// ═══════════════════════════════ backward (tcgen05) ═══════════════════════════════
// Two kernels, no atomics and no fp32 dQ scratch:
//   attn_bwd_kv_tc: CTA = 128 keys of one kv head; loops over the kv group's query heads and the
//     causal query blocks i >= key block. Per block: S^T = K Q^T and dP^T = V dO^T into TMEM;
//     16 element-wise warps (thread = key row, 32 of the 128 query columns; the backward needs no row
//     reduction) form P^T = exp2(S^T*c - LSE) and dS^T = P^T (dP^T - delta) in bf16 shared tiles;
//     dV += P^T dO and dK += dS^T Q accumulate in TMEM; written once at the end.
//   attn_bwd_q_tc: CTA = 128 queries of one head; loops over causal key blocks; recomputes S, dP,
//     forms dS, accumulates dQ += dS K in TMEM; written once (bf16) into dqkv.
// Every tile is loaded once in the 128-byte-swizzled [rows][64-column chunk] layout; the same bytes
// serve as the K-major operand of one product and the MN-major operand of the other (Q, dO, K, and
// the P^T / dS^T tiles, whose row-major [key][query] layout is also dS as an MN-major A operand).
namespace {

constexpr int BW_EW_WARPS = 16;
constexpr int BW_THREADS = 64 + 32 * BW_EW_WARPS;  // warp 0 TMA, warp 1 MMA, warps 2..17 element-wise

// With two operand stages the MMA warp issues S/dP of the next block as soon as the element-wise
// warps have read this block's S/dP out of TMEM, before this block's dV/dK (or dQ) products: the
// tensor cores then work while P / dS of the next block are formed.
template <int D>
struct KVCfg {
  static constexpr int ST = (D == 64) ? 2 : 1;  // Q / dO stages
  static constexpr bool EARLY = ST >= 2;
  static constexpr int T = 128 * D * 2;         // one [128][D] bf16 tile
  static constexpr int PT = 128 * 128 * 2;
  static constexpr int SMEM = 2 * T + ST * 2 * T + 2 * PT + ST * 2 * 512 + 256;
};

template <int D>
struct QCfg {
  static constexpr int ST = (D == 64) ? 2 : 1;  // K / V stages
  static constexpr bool EARLY = ST >= 2;
  static constexpr int T = 128 * D * 2;
  static constexpr int PT = 128 * 128 * 2;
  static constexpr int SMEM = 2 * T + ST * 2 * T + PT + 256;
};

// K-major descriptor of K-step k (16 elements) in a [128 rows][D] swizzled tile made of 64-wide chunks.
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int k) {
  return umma_smem_desc_sw128(base + (k >> 2) * (128 * 128) + (k & 3) * 32, 16, 1024);
}
// MN-major descriptor of K-step k (16 rows) of the same tile used with its columns as the N dimension.
__device__ __forceinline__ uint64_t mndesc(uint32_t base, int k) {
  return umma_smem_desc_sw128(base + k * 2048, 128 * 128, 1024);
}

struct WarpWait {
  volatile int* abort_flag;
  int lane;
  __device__ bool operator()(uint64_t* bb, uint32_t par, int site) const {
    int okl = 1;
    if (lane == 0) okl = mbar_wait_bounded(bb, par, DT_ERR_TIMEOUT_TMEM, site, abort_flag) ? 1 : 0;
    okl = __shfl_sync(0xffffffffu, okl, 0);
    __syncwarp();
    return okl != 0;
  }
};

// One arrival per warp on a barrier initialised with the element-wise warp count.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// Store 32 packed bf16 pairs' worth (32 columns) of row r into a [128 rows][2 x 64-column] 128-byte-
// swizzled tile at column group cg (0..3).
__device__ __forceinline__ void store_row32(uint8_t* tile, int r, int cg, const uint32_t (&v)[16]) {
  uint8_t* row = tile + (cg >> 1) * (128 * 128) + r * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c)
    *reinterpret_cast<uint4*>(row + ((((cg & 1) << 2) + c) ^ (r & 7)) * 16) =
        make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// kv kernel, 32 query columns of one key row: P^T = exp2(S^T*c - LSE*log2e), dS^T = P^T (dP^T - delta),
// with LSE / delta per column (from shared memory). Columns e with !(lo <= e < hi) are zero (MASK).
template <bool MASK>
__device__ __forceinline__ void kv_block_math(const uint32_t (&sv)[32], const uint32_t (&dv)[32], const float* lse,
                                              const float* del, float sl2, int lo, int hi, uint32_t (&pk)[16],
                                              uint32_t (&dk)[16]) {
  const uint64_t c2 = f2_pack(sl2, sl2), m2 = f2_pack(-LOG2E_F, -LOG2E_F);
  const float4* l4 = reinterpret_cast<const float4*>(lse);
  const float4* d4 = reinterpret_cast<const float4*>(del);
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    const float4 l = l4[v], dl = d4[v];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int e = 4 * v + 2 * h2;
      const uint64_t nl = f2_mul(h2 ? f2_pack(l.z, l.w) : f2_pack(l.x, l.y), m2);
      const float2 x = f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), c2, nl));
      float p0 = ex2_approx(x.x), p1 = ex2_approx(x.y);
      const uint64_t dd = f2_sub(f2_pack(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])),
                                 h2 ? f2_pack(dl.z, dl.w) : f2_pack(dl.x, dl.y));
      float2 ds = f2_unpack(f2_mul(f2_pack(p0, p1), dd));
      if (MASK) {
        const bool v0 = (e >= lo) && (e < hi), v1 = (e + 1 >= lo) && (e + 1 < hi);
        p0 = v0 ? p0 : 0.f;
        ds.x = v0 ? ds.x : 0.f;
        p1 = v1 ? p1 : 0.f;
        ds.y = v1 ? ds.y : 0.f;
      }
      pk[e / 2] = pack_bf16(p0, p1);
      dk[e / 2] = pack_bf16(ds.x, ds.y);
    }
  }
}

// q kernel, 32 key columns of one query row: dS = exp2(S*c - LSE*log2e) (dP - delta); LSE / delta are
// this row's. Columns e >= hi are zero (MASK).
template <bool MASK>
__device__ __forceinline__ void q_block_math(const uint32_t (&sv)[32], const uint32_t (&dv)[32], float sl2,
                                             float nlse2, float dlt, int hi, uint32_t (&dk)[16]) {
  const uint64_t c2 = f2_pack(sl2, sl2), nl = f2_pack(nlse2, nlse2), d2 = f2_pack(dlt, dlt);
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const float2 x = f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), c2, nl));
    const float p0 = ex2_approx(x.x), p1 = ex2_approx(x.y);
    const uint64_t dd = f2_sub(f2_pack(__uint_as_float(dv[e]), __uint_as_float(dv[e + 1])), d2);
    float2 ds = f2_unpack(f2_mul(f2_pack(p0, p1), dd));
    if (MASK) {
      ds.x = (e < hi) ? ds.x : 0.f;
      ds.y = (e + 1 < hi) ? ds.y : 0.f;
    }
    dk[e / 2] = pack_bf16(ds.x, ds.y);
  }
}

// bf16 store of `n` (16 or 32) fp32 TMEM columns (times mul) of this thread's lane to dst.
__device__ __forceinline__ void tmem_row_to_bf16(uint32_t taddr, int n, float mul, bool valid,
                                                 __nv_bfloat16* dst) {
  for (int c0 = 0; c0 < n; c0 += 16) {
    uint32_t o[16];
    tmem_ld_32x32b_x16(taddr + c0, o);
    tmem_ld_wait();
    if (valid) {
#pragma unroll
      for (int v = 0; v < 2; ++v) {
        uint4 w;
        w.x = pack_bf16(__uint_as_float(o[8 * v + 0]) * mul, __uint_as_float(o[8 * v + 1]) * mul);
        w.y = pack_bf16(__uint_as_float(o[8 * v + 2]) * mul, __uint_as_float(o[8 * v + 3]) * mul);
        w.z = pack_bf16(__uint_as_float(o[8 * v + 4]) * mul, __uint_as_float(o[8 * v + 5]) * mul);
        w.w = pack_bf16(__uint_as_float(o[8 * v + 6]) * mul, __uint_as_float(o[8 * v + 7]) * mul);
        *reinterpret_cast<uint4*>(dst + c0 + 8 * v) = w;
      }
    }
  }
}

template <int D>
__global__ void __launch_bounds__(BW_THREADS, 1)
attn_bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
                      const __grid_constant__ CUtensorMap tmLSE, const __grid_constant__ CUtensorMap tmDEL,
                      __nv_bfloat16* __restrict__ dqkv, int B, int T, int nh, int nkv, float scale) {
  using C = KVCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 599);
    return;
  }
  uint8_t* sK = smem_raw;
  uint8_t* sV = sK + C::T;
  uint8_t* sQ = sV + C::T;                  // [ST][T]
  uint8_t* sDO = sQ + C::ST * C::T;         // [ST][T]
  uint8_t* sP = sDO + C::ST * C::T;         // P^T  [128 keys][128 q]
  uint8_t* sDS = sP + C::PT;                // dS^T [128 keys][128 q]
  float* sLSE = reinterpret_cast<float*>(sDS + C::PT);  // [ST][128]
  float* sDEL = sLSE + C::ST * 128;                     // [ST][128]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sDEL + C::ST * 128);
  uint64_t* kv_full = bar;
  uint64_t* qd_full = bar + 1;   // [2]
  uint64_t* qd_empty = bar + 3;  // [2]
  uint64_t* sdp_full = bar + 5;
  uint64_t* s_free = bar + 6;
  uint64_t* p_full = bar + 7;
  uint64_t* mm_done = bar + 8;
  uint64_t* drain = bar + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (T + 127) / 128;
  const int kb = blockIdx.x % nkb;  // key block 0 has the most query blocks: scheduled first
  const int bg = blockIdx.x / nkb;
  const int g = bg % nkv, b = bg / nkv;
  const int G = nh / nkv;
  const int nqb = nkb;
  const int iters = G * (nqb - kb);

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&qd_full[i], 1); mbar_init(&qd_empty[i], 1); }
    mbar_init(sdp_full, 1);
    mbar_init(s_free, BW_EW_WARPS);
    mbar_init(p_full, BW_EW_WARPS);
    mbar_init(mm_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(kv_full, 2 * C::T);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(sK + c * (128 * 128), &tmQKV, kv_full, (nh + g) * D + 64 * c, kb * 128, b);
        tma_load_3d(sV + c * (128 * 128), &tmQKV, kv_full, (nh + nkv + g) * D + 64 * c, kb * 128, b);
      }
      for (int it = 0; it < iters; ++it) {
        const int hh = it / (nqb - kb), i = kb + it % (nqb - kb), h = g * G + hh;
        const int st = it % C::ST;
        if (it >= C::ST &&
            !mbar_wait_bounded(&qd_empty[st], ((it / C::ST) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 500, abort_flag))
          break;
        mbar_arrive_expect_tx(&qd_full[st], 2 * C::T + 2 * 512);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sQ + st * C::T + c * (128 * 128), &tmQKV, &qd_full[st], h * D + 64 * c, i * 128, b);
          tma_load_3d(sDO + st * C::T + c * (128 * 128), &tmDO, &qd_full[st], h * D + 64 * c, i * 128, b);
        }
        tma_load_2d(sLSE + st * 128, &tmLSE, &qd_full[st], i * 128, b * nh + h);
        tma_load_2d(sDEL + st * 128, &tmDEL, &qd_full[st], i * 128, b * nh + h);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSS = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idKD = umma_idesc_bf16(128, D, 0, 1);
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aP = smem_u32(sP), aDS = smem_u32(sDS);
      bool issued = false;
      // S^T = K Q^T and dP^T = V dO^T of block `it`
      auto issue_sdp = [&](int it) -> bool {
        const int st = it % C::ST;
        if (!mbar_wait_bounded(&qd_full[st], (it / C::ST) & 1, DT_ERR_TIMEOUT_FULL, 511, abort_flag)) return false;
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ + st * C::T), aDO = smem_u32(sDO + st * C::T);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tS, kdesc(aK, k), kdesc(aQ, k), idSS, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tDP, kdesc(aV, k), kdesc(aDO, k), idSS, k > 0 ? 1u : 0u);
        issued = true;
        umma_commit(sdp_full);
        return true;
      };
      bool ok = mbar_wait_bounded(kv_full, 0, DT_ERR_TIMEOUT_FULL, 510, abort_flag);
      if (ok && C::EARLY && iters > 0) ok = issue_sdp(0);
      for (int it = 0; it < iters && ok; ++it) {
        const int st = it % C::ST;
        if (!C::EARLY) {
          if (it > 0 && !mbar_wait_bounded(s_free, (it - 1) & 1, DT_ERR_TIMEOUT_TMEM, 512, abort_flag)) { ok = false; break; }
          if (!issue_sdp(it)) { ok = false; break; }
        } else if (it + 1 < iters) {
          if (!mbar_wait_bounded(s_free, it & 1, DT_ERR_TIMEOUT_TMEM, 512, abort_flag)) { ok = false; break; }
          if (!issue_sdp(it + 1)) { ok = false; break; }
        }
        if (!mbar_wait_bounded(p_full, it & 1, DT_ERR_TIMEOUT_FULL, 513, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aQ = smem_u32(sQ + st * C::T), aDO = smem_u32(sDO + st * C::T);
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tDV, kdesc(aP, k), mndesc(aDO, k), idKD, (it > 0 || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tDK, kdesc(aDS, k), mndesc(aQ, k), idKD, (it > 0 || k > 0) ? 1u : 0u);
        umma_commit(mm_done);
        umma_commit(&qd_empty[st]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    // ───── element-wise warps: thread = key row r, query columns [cg*32, cg*32+32) ─────
    const int ew = warp - 2, quad = warp & 3, cg = ew >> 2;
    const int r = quad * 32 + lane;
    const int key = kb * 128 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = scale * LOG2E_F;
    const bool edge_k = (kb + 1) * 128 > T;
    WarpWait wwait{abort_flag, lane};
    bool ok = true;
    for (int it = 0; it < iters; ++it) {
      const int i = kb + it % (nqb - kb);
      const int st = it % C::ST;
      if (!wwait(sdp_full, it & 1, 520)) { ok = false; break; }
      tc_fence_after();
      uint32_t pk[16], dk[16];
      {
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(tS + lane_off + cg * 32, sv);
        tmem_ld_32x32b_x32(tDP + lane_off + cg * 32, dv);
        tmem_ld_wait();
        const float* lse_s = sLSE + st * 128 + cg * 32;
        const float* del_s = sDEL + st * 128 + cg * 32;
        if (i == kb || edge_k || (i + 1) * 128 > T) {
          const int qbase = i * 128 + cg * 32;
          const int lo = key - qbase, hi = key < T ? T - qbase : 0;  // valid columns: lo <= e < hi
          kv_block_math<true>(sv, dv, lse_s, del_s, sl2, lo, hi, pk, dk);
        } else {
          kv_block_math<false>(sv, dv, lse_s, del_s, sl2, 0, 32, pk, dk);
        }
      }
      tc_fence_before();
      warp_arrive(s_free, lane);
      // the previous block's dV / dK products must be done reading the P^T / dS^T tiles
      if (it > 0 && !wwait(mm_done, (it - 1) & 1, 521)) { ok = false; break; }
      store_row32(sP, r, cg, pk);
      store_row32(sDS, r, cg, dk);
      fence_proxy_async_smem();
      warp_arrive(p_full, lane);
    }
    // epilogue: dK (scaled) and dV rows of this key block, D/4 columns per thread
    if (ok && wwait(mm_done, (iters - 1) & 1, 522)) {
      tc_fence_after();
      const long long W = (long long)(nh + 2 * nkv) * D;
      __nv_bfloat16* krow = dqkv + ((long long)b * T + key) * W + (nh + g) * D + cg * (D / 4);
      __nv_bfloat16* vrow = dqkv + ((long long)b * T + key) * W + (nh + nkv + g) * D + cg * (D / 4);
      tmem_row_to_bf16(tDK + lane_off + cg * (D / 4), D / 4, scale, key < T, krow);
      tmem_row_to_bf16(tDV + lane_off + cg * (D / 4), D / 4, 1.f, key < T, vrow);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <int D>
__global__ void __launch_bounds__(BW_THREADS, 1)
attn_bwd_q_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
                     const float* __restrict__ lse, const float* __restrict__ delta, __nv_bfloat16* __restrict__ dqkv,
                     int B, int T, int nh, int nkv, float scale) {
  using C = QCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 699);
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sDO = sQ + C::T;
  uint8_t* sK = sDO + C::T;         // [ST][T]
  uint8_t* sV = sK + C::ST * C::T;  // [ST][T]
  uint8_t* sDS = sV + C::ST * C::T; // dS [128 q][128 keys]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sDS + C::PT);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;   // [2]
  uint64_t* kv_empty = bar + 3;  // [2]
  uint64_t* sdp_full = bar + 5;
  uint64_t* s_free = bar + 6;
  uint64_t* p_full = bar + 7;
  uint64_t* mm_done = bar + 8;
  uint64_t* drain = bar + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (T + 127) / 128;
  const int qb = nqb - 1 - (blockIdx.x % nqb);  // long (late) query blocks first
  const int bh = blockIdx.x / nqb;
  const int h = bh % nh, b = bh / nh;
  const int g = h / (nh / nkv);
  const int nkb = qb + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    mbar_init(sdp_full, 1);
    mbar_init(s_free, BW_EW_WARPS);
    mbar_init(p_full, BW_EW_WARPS);
    mbar_init(mm_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 128, tDQ = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(q_full, 2 * C::T);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(sQ + c * (128 * 128), &tmQKV, q_full, h * D + 64 * c, qb * 128, b);
        tma_load_3d(sDO + c * (128 * 128), &tmDO, q_full, h * D + 64 * c, qb * 128, b);
      }
      for (int j = 0; j < nkb; ++j) {
        const int st = j % C::ST;
        if (j >= C::ST &&
            !mbar_wait_bounded(&kv_empty[st], ((j / C::ST) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 600, abort_flag))
          break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::T);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sK + st * C::T + c * (128 * 128), &tmQKV, &kv_full[st], (nh + g) * D + 64 * c, j * 128, b);
          tma_load_3d(sV + st * C::T + c * (128 * 128), &tmQKV, &kv_full[st], (nh + nkv + g) * D + 64 * c, j * 128, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSS = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idQD = umma_idesc_bf16(128, D, 0, 1);
      const uint32_t aQ = smem_u32(sQ), aDO = smem_u32(sDO), aDS = smem_u32(sDS);
      bool issued = false;
      // S = Q K^T and dP = dO V^T of key block j
      auto issue_sdp = [&](int j) -> bool {
        const int st = j % C::ST;
        if (!mbar_wait_bounded(&kv_full[st], (j / C::ST) & 1, DT_ERR_TIMEOUT_FULL, 611, abort_flag)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * C::T), aV = smem_u32(sV + st * C::T);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tS, kdesc(aQ, k), kdesc(aK, k), idSS, k > 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tDP, kdesc(aDO, k), kdesc(aV, k), idSS, k > 0 ? 1u : 0u);
        issued = true;
        umma_commit(sdp_full);
        return true;
      };
      bool ok = mbar_wait_bounded(q_full, 0, DT_ERR_TIMEOUT_FULL, 610, abort_flag);
      if (ok && C::EARLY) ok = issue_sdp(0);
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j % C::ST;
        if (!C::EARLY) {
          if (j > 0 && !mbar_wait_bounded(s_free, (j - 1) & 1, DT_ERR_TIMEOUT_TMEM, 612, abort_flag)) { ok = false; break; }
          if (!issue_sdp(j)) { ok = false; break; }
        } else if (j + 1 < nkb) {
          if (!mbar_wait_bounded(s_free, j & 1, DT_ERR_TIMEOUT_TMEM, 612, abort_flag)) { ok = false; break; }
          if (!issue_sdp(j + 1)) { ok = false; break; }
        }
        if (!mbar_wait_bounded(p_full, j & 1, DT_ERR_TIMEOUT_FULL, 613, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + st * C::T);
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16(tDQ, kdesc(aDS, k), mndesc(aK, k), idQD, (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(mm_done);
        umma_commit(&kv_empty[st]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    // ───── element-wise warps: thread = query row r, key columns [cg*32, cg*32+32) ─────
    const int ew = warp - 2, quad = warp & 3, cg = ew >> 2;
    const int r = quad * 32 + lane;
    const int q = qb * 128 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = scale * LOG2E_F;
    const int Tp = (T + 3) & ~3;
    const long long ridx = ((long long)b * nh + h) * Tp + q;
    const float nlse2 = (q < T) ? -lse[ridx] * LOG2E_F : 0.f;
    const float dlt = (q < T) ? delta[ridx] : 0.f;
    const bool edge_q = (qb + 1) * 128 > T;
    WarpWait wwait{abort_flag, lane};
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (!wwait(sdp_full, j & 1, 620)) { ok = false; break; }
      tc_fence_after();
      uint32_t dk[16];
      {
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(tS + lane_off + cg * 32, sv);
        tmem_ld_32x32b_x32(tDP + lane_off + cg * 32, dv);
        tmem_ld_wait();
        if (j == qb || edge_q || (j + 1) * 128 > T) {
          const int kbase = j * 128 + cg * 32;
          const int hi = q < T ? min(q - kbase + 1, T - kbase) : 0;  // valid columns: e < hi
          q_block_math<true>(sv, dv, sl2, nlse2, dlt, hi, dk);
        } else {
          q_block_math<false>(sv, dv, sl2, nlse2, dlt, 32, dk);
        }
      }
      tc_fence_before();
      warp_arrive(s_free, lane);
      if (j > 0 && !wwait(mm_done, (j - 1) & 1, 621)) { ok = false; break; }
      store_row32(sDS, r, cg, dk);
      fence_proxy_async_smem();
      warp_arrive(p_full, lane);
    }
    if (ok && wwait(mm_done, (nkb - 1) & 1, 622)) {
      tc_fence_after();
      const long long W = (long long)(nh + 2 * nkv) * D;
      __nv_bfloat16* qrow = dqkv + ((long long)b * T + q) * W + h * D + cg * (D / 4);
      tmem_row_to_bf16(tDQ + lane_off + cg * (D / 4), D / 4, scale, q < T, qrow);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// fp32 [rows, Tp] map with a {128, 1} box (LSE / delta slices of one query block).
int rowvec_map(CUtensorMap* m, const float* p, long long rows, long long Tp) {
  if (!g_enc) return -2;
  cuuint64_t dims[2] = {(cuuint64_t)Tp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(Tp * 4)};
  cuuint32_t box[2] = {128, 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

template <int D>
int bwd_tc_launch(const void* qkv, const void* dout, const float* lse, const float* delta, void* dqkv, int B, int T,
                  int nh, int nkv, float scale, cudaStream_t st) {
  long long W = (long long)(nh + 2 * nkv) * D;
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(lse) |
       reinterpret_cast<uintptr_t>(delta)) & 15)
    return -10;
  const long long Tp = (T + 3) & ~3;
  CUtensorMap mq, mdo, ml, md;
  int rc = qkv_map(&mq, qkv, B, T, W);
  if (!rc) rc = qkv_map(&mdo, dout, B, T, (long long)nh * D);
  if (!rc) rc = rowvec_map(&ml, lse, (long long)B * nh, Tp);
  if (!rc) rc = rowvec_map(&md, delta, (long long)B * nh, Tp);
  if (rc) return rc;
  static bool set = false;
  if (!set) {
    DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_kv_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, KVCfg<D>::SMEM));
    DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_q_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, QCfg<D>::SMEM));
    set = true;
  }
  const int nb = (T + 127) / 128;
  auto dq = reinterpret_cast<__nv_bfloat16*>(dqkv);
  attn_bwd_kv_tc_kernel<D><<<B * nkv * nb, BW_THREADS, KVCfg<D>::SMEM, st>>>(mq, mdo, ml, md, dq, B, T, nh, nkv, scale);
  DT_CUDA_RET(cudaGetLastError());
  attn_bwd_q_tc_kernel<D><<<B * nh * nb, BW_THREADS, QCfg<D>::SMEM, st>>>(mq, mdo, lse, delta, dq, B, T, nh, nkv, scale);
  return (int)cudaGetLastError();
}

}  // namespace

// tcgen05 backward (d = 64 / 128). `delta` must already hold rowsum(dO * O) (dt_attn_bwd_delta).
DT_API int dt_attn_bwd_tc(const void* qkv, const void* dout, const float* lse, const float* delta, void* dqkv, int B,
                          int T, int nh, int nkv, int D, float scale, cudaStream_t st) {
  if (nh % nkv) return -10;
  if (D == 64) return bwd_tc_launch<64>(qkv, dout, lse, delta, dqkv, B, T, nh, nkv, scale, st);
  if (D == 128) return bwd_tc_launch<128>(qkv, dout, lse, delta, dqkv, B, T, nh, nkv, scale, st);
  return -11;
}
