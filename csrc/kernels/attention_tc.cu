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
      if (q < T) lse[((long long)b * nh + h) * T + q] = (m_run + log2f(l_run)) * LN2_F;
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
