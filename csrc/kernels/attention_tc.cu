// Causal GQA flash attention on the 5th-generation tensor cores (tcgen05 + TMEM), d = 64 / 128.
//
// Same contract as the mma.sync kernels in attention.cu (q/k/v read from the fused QKV activation,
// query head h uses kv head h / (nh/nkv), out [B*T, nh*D] bf16, lse [B, nh, Tp] fp32 natural log with
// Tp = T rounded up to a multiple of 4 so every row starts 16-byte aligned).
//
// Cost model behind the layouts (measured on B200): a tcgen05.mma with M = 128 costs the tensor core
// about N/2 clocks, but a single issuing thread does not issue much faster than one per ~50 clocks, so
// products are kept N = 128 wide where the shapes allow, the issue loops only add constants to
// precomputed descriptors, and two CTAs share an SM where TMEM allows (two issuers). The softmax side
// is bound by the exp2 unit (16 results / clock / SM).
//
// Forward. Persistent: CTAS x SMs CTAs loop over tiles of 128 query rows of one (batch, head), heaviest
// (longest causal) query blocks first; the next tile's Q (double-buffered) and K/V loads and its first
// product overlap the current tile's last softmax and epilogue. 10 warps:
//   warp 0     TMA producer: Q once, then K/V tiles of 128 keys into a 2-stage ring (3-D tensor map
//              [B, T, W] so rows past T are zero-filled per sequence; no cluster multicast)
//   warp 1     single-thread tcgen05.mma issuer: S = Q K^T (N = 128) into TMEM; O += P V with P a TMEM
//              A operand and V an MN-major shared operand. S of block j+1 is issued as soon as the
//              softmax warps have read S of block j, before P V of block j.
//   warps 2-9  softmax: two threads per query row (TMEM lane), 64 columns each; the row max is
//              exchanged through shared memory once per block. The running
//              max is only raised when it grows by more than 8 (log2 units); O in TMEM is rescaled
//              (tcgen05.ld/st) only then, otherwise P is taken against the stale max (values stay
//              <= 2^8, exact after normalisation). The pair exchanges through per-quarter mbarriers
//              (bounded waits), not a named barrier, so a warp that gives up cannot strand its partner.
// TMEM: S [0,128), O [128,128+D), P (bf16 pairs) [128+D, 192+D): 256 columns at d = 64, so two CTAs
// share an SM and one CTA's softmax overlaps the other's products. Every mbarrier wait is bounded.
#include "common.cuh"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

// Optional event trace (build with -DDT_ATTN_TRACE): SM clock of each pipeline event of one CTA,
// slot = event * 64 + iteration, read back by a profiling harness.
#ifdef DT_ATTN_TRACE
__device__ unsigned long long g_attn_trace[8 * 64];
__device__ int g_attn_trace_block;
__device__ unsigned long long g_cta_trace[4 * 65536];  // per CTA: start ns, setup-done ns, end ns, SM id
__device__ __forceinline__ void cta_trace(int slot) {
  if (threadIdx.x == 0 && blockIdx.x < 65536) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    g_cta_trace[blockIdx.x * 4 + slot] = t;
    if (slot == 2) {
      unsigned sm;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
      g_cta_trace[blockIdx.x * 4 + 3] = sm;
    }
  }
}
#define CTA_TRACE(slot) cta_trace(slot)
#define ATTN_TRACE(ev, it)                                  \
  do {                                                      \
    if ((int)blockIdx.x == g_attn_trace_block && (it) < 64) \
      g_attn_trace[(ev) * 64 + (it)] = clock64();           \
  } while (0)
#else
#define ATTN_TRACE(ev, it) \
  do {                     \
  } while (0)
#define CTA_TRACE(slot) \
  do {                  \
  } while (0)
#endif

namespace {

constexpr int BQ = 128, BKV = 128;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float LN2_F = 0.6931471805599453f;
constexpr float RESCALE_THRESHOLD = 8.0f;

// Descriptor offsets (in 16-byte units) of K-step k within a [128 rows][D] swizzled tile of 64-wide
// chunks: K-major (16 elements along the row) and MN-major (16 rows) use.
__host__ __device__ constexpr uint64_t koff(int k) { return (uint64_t)(((k >> 2) * (128 * 128) + (k & 3) * 32) >> 4); }
__host__ __device__ constexpr uint64_t mnoff(int k) { return (uint64_t)((k * 2048) >> 4); }
__device__ __forceinline__ uint64_t kdesc0(uint32_t base) { return umma_smem_desc_sw128(base, 16, 1024); }
__device__ __forceinline__ uint64_t mndesc0(uint32_t base) { return umma_smem_desc_sw128(base, 128 * 128, 1024); }

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

// One arrival per warp on a barrier initialised with the number of arriving warps.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// bf16 store of `n` (a multiple of 16) fp32 TMEM columns (times mul) of this thread's lane to dst.
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

// In-place scale of `n` (a multiple of 16) fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_row_scale(uint32_t taddr, int n, float mul) {
  for (int c0 = 0; c0 < n; c0 += 16) {
    uint32_t o[16];
    tmem_ld_32x32b_x16(taddr + c0, o);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * mul);
    tmem_st_32x32b_x16(taddr + c0, o);
  }
  tmem_st_wait();
}

constexpr int FWD_SM_WARPS = 8;                    // softmax warps: two per TMEM lane quarter
constexpr int FWD_THREADS = 64 + 32 * FWD_SM_WARPS;

template <int D>
struct FCfg {
  static constexpr int CTAS = (D == 64) ? 2 : 1;   // CTAs per SM
  static constexpr int ST = 2;                     // K / V stages
  static constexpr int TT = 128 * D * 2;           // one [128][D] bf16 tile
  // Q double-buffered (the next tile's Q arrives while this tile runs) + K/V ring + max/sum exchange
  static constexpr int SMEM = 2 * TT + ST * 2 * TT + 4 * 128 * 4 + 2 * 128 * 4 + 256;
  static constexpr int TMEM_COLS = (D == 64) ? 256 : 512;
  static constexpr int C_O = 128, C_P = 128 + D;
  static_assert(C_P + 64 <= TMEM_COLS, "forward TMEM budget");
};
static_assert(2 * (FCfg<64>::SMEM + 1024) <= 233472 && FCfg<128>::SMEM <= 232448, "forward shared memory");

// Work unit (tile) t of the forward: heaviest query blocks first across all (batch, head) pairs
// (a longest-processing-time-first order for the persistent CTAs).
struct FwdTile {
  int b, h, qb, g, nkb;
};
__device__ __forceinline__ FwdTile fwd_tile(int t, int B, int nh, int nkv, int nqb) {
  FwdTile w;
  const int bh_count = B * nh;
  w.qb = nqb - 1 - t / bh_count;
  const int bh = t % bh_count;
  w.h = bh % nh;
  w.b = bh / nh;
  w.g = w.h / (nh / nkv);
  w.nkb = w.qb + 1;  // causal: key blocks 0..qb (BKV == BQ)
  return w;
}

// Persistent forward: a grid of CTAS x SMs CTAs, each looping over tiles blockIdx.x, +gridDim.x, ...
// All warps walk the same tile sequence; barrier phases follow a global key-block counter `jg` (K/V ring,
// S / P / O hand-offs, max exchange) and a tile counter `tl` (Q buffers, sum exchange), so the next
// tile's Q and K/V loads and its first S = Q K^T overlap this tile's last softmax and epilogue.
template <int D>
__global__ void __launch_bounds__(FWD_THREADS, FCfg<D>::CTAS)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, __nv_bfloat16* __restrict__ out,
                   float* __restrict__ lse, int B, int T, int nh, int nkv, float scale) {
  using C = FCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  CTA_TRACE(0);
  if (smem_u32(smem_raw) & 1023) {  // uniform across the CTA; nothing allocated yet
    if (threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 499);
    return;
  }
  uint8_t* sQ = smem_raw;               // [2][TT]
  uint8_t* sK = sQ + 2 * C::TT;         // [ST][TT]
  uint8_t* sV = sK + C::ST * C::TT;     // [ST][TT]
  float* sMax = reinterpret_cast<float*>(sV + C::ST * C::TT);  // [2 parity][2 halves][128 rows]
  float* sL = sMax + 4 * 128;                                  // [2 halves][128 rows]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sL + 2 * 128);
  uint64_t* q_full = bar;                // [2]
  uint64_t* q_empty = bar + 2;           // [2]
  // K and V have rings of their own: a K stage is free once its S = Q K^T has completed, a V stage once
  // its P V has, so the next K loads start about one softmax phase earlier than with shared stages
  uint64_t* kv_full = bar + 4;           // [ST] K
  uint64_t* kv_empty = bar + 4 + C::ST;  // [ST] K
  uint64_t* v_full = bar + 4 + 2 * C::ST;
  uint64_t* v_empty = bar + 4 + 3 * C::ST;
  uint64_t* s_full = bar + 4 + 4 * C::ST;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_full + 2;
  uint64_t* pv_done = s_full + 3;
  uint64_t* drain = s_full + 4;
  uint64_t* xch = s_full + 5;  // [4 quarters][3]: row-max exchange (block parity 0 / 1), row-sum exchange
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 5 + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (T + BQ - 1) / BQ;
  const int ntiles = B * nh * nqb;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], 1); }
    for (int i = 0; i < C::ST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, FWD_SM_WARPS);
    mbar_init(p_full, FWD_SM_WARPS);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 12; ++i) mbar_init(&xch[i], 2);
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
  const uint32_t tS = tmem, tO = tmem + C::C_O, tP = tmem + C::C_P;
  CTA_TRACE(1);

  if (warp == 0) {
    // ───── TMA producer: per tile its Q (double buffer), then its K blocks into the K ring; each block's
    // V follows one step behind its K (V is needed only by P V, after that block's softmax) ─────
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      int nk = 0, nv = 0, tl = 0;  // K / V loads issued, tile counter
      int v_x = 0, v_j = 0, v_b = 0;
      bool ok = true, v_pending = false;
      auto load_v = [&]() -> bool {  // V of global block nv at (column v_x, key block v_j, batch v_b)
        const int st = nv % C::ST;
        if (nv >= C::ST &&
            !mbar_wait_bounded(&v_empty[st], ((nv / C::ST) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 402, abort_flag))
          return false;
        mbar_arrive_expect_tx(&v_full[st], C::TT);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sV + st * C::TT + c * (BKV * 128), &tmQKV, &v_full[st], v_x + 64 * c, v_j * BKV, v_b);
        ++nv;
        v_pending = false;
        return true;
      };
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tl) {
        const FwdTile w = fwd_tile(t, B, nh, nkv, nqb);
        const int qbuf = tl & 1;
        if (tl >= 2 &&
            !mbar_wait_bounded(&q_empty[qbuf], ((tl >> 1) - 1) & 1, DT_ERR_TIMEOUT_EMPTY, 401, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&q_full[qbuf], C::TT);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sQ + qbuf * C::TT + c * (BQ * 128), &tmQKV, &q_full[qbuf], w.h * D + 64 * c, w.qb * BQ, w.b);
        const int xk = (nh + w.g) * D, xv = (nh + nkv + w.g) * D;
        for (int j = 0; j < w.nkb; ++j) {
          const int st = nk % C::ST;
          if (nk >= C::ST &&
              !mbar_wait_bounded(&kv_empty[st], ((nk / C::ST) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 400, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], C::TT);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_3d(sK + st * C::TT + c * (BKV * 128), &tmQKV, &kv_full[st], xk + 64 * c, j * BKV, w.b);
          ++nk;
          if (v_pending && !load_v()) { ok = false; break; }
          v_x = xv; v_j = j; v_b = w.b;
          v_pending = true;
        }
      }
      if (ok && v_pending) ok = load_v();
      if (!ok) {
        // an aborted run: let the loads already issued land before the CTA exits (bounded)
        uint64_t t0 = dt_globaltimer();
        for (int k = (nk > C::ST ? nk - C::ST : 0); k < nk; ++k)
          while (!mbar_try_wait(&kv_full[k % C::ST], (k / C::ST) & 1) && dt_globaltimer() - t0 < 20000000ull) {}
        for (int k = (nv > C::ST ? nv - C::ST : 0); k < nv; ++k)
          while (!mbar_try_wait(&v_full[k % C::ST], (k / C::ST) & 1) && dt_globaltimer() - t0 < 20000000ull) {}
        for (int k = (tl > 2 ? tl - 2 : 0); k <= tl && k >= 0; ++k)
          while (!mbar_try_wait(&q_full[k & 1], (k >> 1) & 1) && dt_globaltimer() - t0 < 20000000ull) {}
      }
    }
  } else if (warp == 1) {
    // ───── single-thread tcgen05.mma issuer ─────
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(BQ, BKV, 0, 0);
      constexpr uint32_t idO = umma_idesc_bf16(BQ, D, 0, 1);
      constexpr uint64_t STG = (uint64_t)(C::TT >> 4);
      const uint64_t dQ0 = kdesc0(smem_u32(sQ)), dK0 = kdesc0(smem_u32(sK)), mV0 = mndesc0(smem_u32(sV));
      bool issued = false;
      // S = Q K^T of global key block jg (of a tile whose Q sits in buffer qbuf, tile counter tl)
      auto issue_s = [&](int jg, int qbuf, int tl, bool first_of_tile) -> bool {
        if (first_of_tile &&
            !mbar_wait_bounded(&q_full[qbuf], (tl >> 1) & 1, DT_ERR_TIMEOUT_FULL, 410, abort_flag))
          return false;
        if (!mbar_wait_bounded(&kv_full[jg % C::ST], (jg / C::ST) & 1, DT_ERR_TIMEOUT_FULL, 411, abort_flag))
          return false;
        tc_fence_after();
        const uint64_t qq = dQ0 + (uint64_t)qbuf * STG;
        const uint64_t kk = dK0 + (uint64_t)(jg % C::ST) * STG;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tS, qq + koff(k), kk + koff(k), idS, k > 0 ? 1u : 0u);
        umma_commit(s_full);
        umma_commit(&kv_empty[jg % C::ST]);  // this K stage is free once S has read it
        ATTN_TRACE(0, jg);
        issued = true;
        return true;
      };
      int jg = 0, tl = 0;
      int t = blockIdx.x;
      bool ok = t < ntiles;
      FwdTile w = fwd_tile(t < ntiles ? t : 0, B, nh, nkv, nqb);
      if (ok) ok = issue_s(0, 0, 0, true);
      for (; t < ntiles && ok; t += gridDim.x, ++tl) {
        const int qbuf = tl & 1;
        const int tn = t + gridDim.x;  // next tile of this CTA
        for (int j = 0; j < w.nkb && ok; ++j, ++jg) {
          const int st = jg % C::ST;
          const bool last = j + 1 == w.nkb;
          if (!last || tn < ntiles) {
            // S of the next key block (this tile's, or the next tile's first) once S(jg) has been read
            if (!mbar_wait_bounded(s_free, jg & 1, DT_ERR_TIMEOUT_TMEM, 412, abort_flag)) { ok = false; break; }
            if (last) umma_commit(&q_empty[qbuf]);  // every S of this tile is issued: its Q may be replaced
            if (!issue_s(jg + 1, last ? qbuf ^ 1 : qbuf, last ? tl + 1 : tl, last)) { ok = false; break; }
          }
          if (!mbar_wait_bounded(p_full, jg & 1, DT_ERR_TIMEOUT_FULL, 413, abort_flag)) { ok = false; break; }
          if (!mbar_wait_bounded(&v_full[st], (jg / C::ST) & 1, DT_ERR_TIMEOUT_FULL, 414, abort_flag)) {
            ok = false;
            break;
          }
          ATTN_TRACE(1, jg);
          tc_fence_after();
          const uint64_t vv = mV0 + (uint64_t)st * STG;
#pragma unroll
          for (int k = 0; k < BKV / 16; ++k)
            umma_bf16_ts(tO, tP + k * 8, vv + mnoff(k), idO, (j > 0 || k > 0) ? 1u : 0u);
          umma_commit(pv_done);
          umma_commit(&v_empty[st]);
        }
        if (tn < ntiles) w = fwd_tile(tn, B, nh, nkv, nqb);
      }
      if (!ok && issued) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    // ───── softmax warps: row r = TMEM lane r, key columns [cg*64, cg*64+64) of each block ─────
    const int sw = warp - 2, quad = warp & 3, cg = sw >> 2;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = scale * LOG2E_F;
    const uint64_t sl2v = f2_pack(sl2, sl2);
    WarpWait wwait{abort_flag, lane};
    bool ok = true;
    int jg = 0, tl = 0;
    for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++tl) {
      const FwdTile w = fwd_tile(t, B, nh, nkv, nqb);
      const int q = w.qb * BQ + r;
      float m_run = -INFINITY, l_part = 0.f;
      for (int j = 0; j < w.nkb; ++j, ++jg) {
        if (!wwait(s_full, jg & 1, 420)) { ok = false; break; }
        if (warp == 2 && lane == 0) ATTN_TRACE(2, jg);
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld_32x32b_x32(tS + lane_off + cg * 64, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld_32x32b_x32(tS + lane_off + cg * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(s_free, lane);
        const int key0 = j * BKV + cg * 64;
        const bool need_mask = (j == w.qb) || (j + 1) * BKV > T;
        // valid columns e < hi (causal key <= q, key < T); rows q >= T have none
        const int hi = need_mask ? (q < T ? min(q - key0 + 1, T - key0) : 0) : 64;
        float mx = -INFINITY;
        if (need_mask) {
#pragma unroll
          for (int e = 0; e < 64; ++e) mx = (e < hi) ? fmaxf(mx, __uint_as_float(sv[e])) : mx;
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e) mx = fmaxf(mx, __uint_as_float(sv[e]));
        }
        // row max over both halves (partner warp: same lane quarter, other column half)
        float* mbuf = sMax + (jg & 1) * 256;
        mbuf[cg * 128 + r] = mx;
        warp_arrive(&xch[quad * 3 + (jg & 1)], lane);
        if (!wwait(&xch[quad * 3 + (jg & 1)], (jg >> 1) & 1, 423)) { ok = false; break; }
        mx = fmaxf(mx, mbuf[(cg ^ 1) * 128 + r]);
        if (warp == 2 && lane == 0) ATTN_TRACE(3, jg);
        const float m_new = mx * sl2;  // -inf when the row has no valid key yet
        // stale-max policy: raise the reference max only when it grows by more than the threshold
        float m_use = m_run;
        bool resc = false;
        if (m_new > m_run + RESCALE_THRESHOLD || m_run == -INFINITY) {
          m_use = m_new;
          resc = (m_run != -INFINITY);
        }
        const float m_safe = (m_use == -INFINITY) ? 0.f : m_use;
        const float alpha = resc ? ex2_approx(m_run - m_use) : 1.f;
        const uint64_t nm = f2_pack(-m_safe, -m_safe);
        uint32_t pk[32];
        uint64_t rs2 = f2_pack(0.f, 0.f);
#pragma unroll
        for (int e = 0; e < 64; e += 2) {
          const float2 x = f2_unpack(f2_fma(f2_pack(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), sl2v, nm));
          float p0 = ex2_approx(x.x), p1 = ex2_approx(x.y);
          if (need_mask) {
            p0 = (e < hi) ? p0 : 0.f;
            p1 = (e + 1 < hi) ? p1 : 0.f;
          }
          rs2 = f2_add(rs2, f2_pack(p0, p1));
          pk[e / 2] = pack_bf16(p0, p1);
        }
        const float2 rs = f2_unpack(rs2);
        l_part = l_part * alpha + (rs.x + rs.y);
        m_run = m_use;
        if (warp == 2 && lane == 0) ATTN_TRACE(4, jg);
        // P and O are busy until the previous P V of this tile has completed (the previous tile's last
        // P V was waited for by its epilogue)
        if (j > 0 && !wwait(pv_done, (jg - 1) & 1, 421)) { ok = false; break; }
        if (warp == 2 && lane == 0) ATTN_TRACE(5, jg);
        tc_fence_after();
        if (j > 0 && __any_sync(0xffffffffu, resc)) tmem_row_scale(tO + lane_off + cg * (D / 2), D / 2, alpha);
        tmem_st_32x32b_x16(tP + lane_off + cg * 32, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
        tmem_st_32x32b_x16(tP + lane_off + cg * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
        tmem_st_wait();
        tc_fence_before();
        warp_arrive(p_full, lane);
        if (warp == 2 && lane == 0) ATTN_TRACE(6, jg);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16 rows of `out` (this half's D/2 columns), lse
      if (!wwait(pv_done, (jg - 1) & 1, 422)) { ok = false; break; }
      tc_fence_after();
      sL[cg * 128 + r] = l_part;
      warp_arrive(&xch[quad * 3 + 2], lane);
      if (!wwait(&xch[quad * 3 + 2], tl & 1, 424)) { ok = false; break; }
      const float l = l_part + sL[(cg ^ 1) * 128 + r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + ((long long)w.b * T + q) * ((long long)nh * D) + w.h * D + cg * (D / 2);
      tmem_row_to_bf16(tO + lane_off + cg * (D / 2), D / 2, inv, q < T, orow);
      if (cg == 0 && q < T) lse[((long long)w.b * nh + w.h) * ((T + 3) & ~3) + q] = (m_run + log2f(l)) * LN2_F;
      // the partner reads sL before either warp writes it for the next tile: the next tile's first
      // max exchange (which both must pass) orders it
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
  CTA_TRACE(2);
}

PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;
std::once_flag g_enc_once;

int qkv_map(CUtensorMap* m, const void* qkv, int B, int T, long long W, int rows = 128) {
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
  cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
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
  const int nqb = (T + BQ - 1) / BQ;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    DT_CUDA_RET(cudaGetDevice(&dev));
    DT_CUDA_RET(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  }
  const long long tiles = (long long)B * nh * nqb;
  const int grid = (int)(tiles < (long long)C::CTAS * sms ? tiles : (long long)C::CTAS * sms);  // persistent
  attn_fwd_tc_kernel<D><<<grid, FWD_THREADS, C::SMEM, st>>>(m, reinterpret_cast<__nv_bfloat16*>(out), lse, B, T, nh,
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
//     causal 128-query blocks. Per block: S^T = K Q^T and dP^T = V dO^T (128 x 128, fp32) into TMEM;
//     16 element-wise warps (thread = key row, 32 of the 128 query columns; the backward needs no row
//     reduction) form P^T = exp2(S^T*c - LSE) and dS^T = P^T (dP^T - delta) as bf16 pairs stored back
//     into the S^T columns the thread has just read; dV += P^T dO and dK += dS^T Q take them as TMEM A
//     operands and accumulate in TMEM; written once at the end.
//   attn_bwd_q_tc: CTA = 128 queries of one head; loops over the causal 128-key blocks; recomputes S
//     and dP (Q and dO held in TMEM as A operands), forms dS in TMEM, accumulates dQ += dS K.
// Products are kept N = 128 wide where the shapes allow (see the cost model at the top). At
// d = 64 S^T is double-buffered in TMEM (columns: S 2 x 128, dP 128, dV 64, dK 64) so the tensor cores
// compute block i+1 while block i's exponentials (16 results / clock / SM) run; at d = 128 the
// accumulators take the room of the second buffer.
// Tiles arrive by TMA in the 128-byte-swizzled [64-column chunk][rows][128 B] layout; the same bytes
// serve as the K-major operand of one product and the MN-major operand of the other (Q, dO, K).


namespace {

constexpr int BW_EW_WARPS = 16;
constexpr int BW_THREADS = 64 + 32 * BW_EW_WARPS;  // warp 0 TMA, warp 1 MMA, warps 2..17 element-wise

template <int D, bool DS = false>
struct KVCfg {
  static constexpr int NSB = (D == 64) ? 2 : 1;  // S^T buffers in TMEM
  static constexpr int ST = (D == 64) ? (DS ? 3 : 4) : 2;   // Q / dO stages
  static constexpr int TT = 128 * D * 2;         // one [128][D] bf16 tile
  static constexpr int DS_BYTES = DS ? 2 * 128 * 128 * 2 : 0;  // two dS^T staging tiles (TMA-stored)
  static constexpr int SMEM = 2 * TT + ST * 2 * TT + ST * 2 * 512 + DS_BYTES + 512;
  // TMEM columns
  static constexpr int C_DP = NSB * 128, C_DV = C_DP + 128, C_DK = C_DV + D;
  static_assert(C_DK + D <= 512, "kv TMEM budget");
};

template <int D>
struct QCfg {
  static constexpr int NSB = (D == 64) ? 2 : 1;  // S buffers in TMEM
  static constexpr int ST = (D == 64) ? 4 : 2;   // K / V stages
  static constexpr int TT = 128 * D * 2;
  static constexpr int SMEM = 2 * TT + ST * 2 * TT + 256;
  static constexpr int C_DP = NSB * 128, C_DQ = C_DP + 128, C_Q = C_DQ + D, C_DO = C_Q + D / 2;
  static_assert(C_DO + D / 2 <= 512, "q TMEM budget");
};

static_assert(KVCfg<64>::SMEM <= 232448 && KVCfg<128>::SMEM <= 232448 && KVCfg<64, true>::SMEM <= 232448,
              "kv backward shared memory");
static_assert(QCfg<64>::SMEM <= 232448 && QCfg<128>::SMEM <= 232448, "q backward shared memory");

// TMEM A operand of K-step k of a bf16 tile written by the element-wise threads: thread group cg holds
// elements [32cg, 32cg+32) as 16 packed columns at buf + 32cg + half*16; K-step k is group k>>1's
// columns (k&1)*8 .. +8.
__device__ __forceinline__ uint32_t pcol(uint32_t buf, int half, int k) {
  return buf + (k >> 1) * 32 + half * 16 + (k & 1) * 8;
}

// Copy row r, elements [cg*D/4, (cg+1)*D/4) of a swizzled [128][D] bf16 shared tile into TMEM as packed
// pairs (column = element / 2) at tdst + lane offset: the tile becomes a TMEM A operand.
template <int D>
__device__ __forceinline__ void tile_row_to_tmem(const uint8_t* tile, int r, int cg, uint32_t tdst) {
#pragma unroll
  for (int u = 0; u < D / 32; u += 2) {
    uint32_t v[8];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      const int e0 = cg * (D / 4) + (u + w) * 8;
      const uint4 x = *reinterpret_cast<const uint4*>(tile + (e0 >> 6) * (128 * 128) + r * 128 +
                                                      ((((e0 & 63) >> 3) ^ (r & 7)) << 4));
      v[4 * w] = x.x;
      v[4 * w + 1] = x.y;
      v[4 * w + 2] = x.z;
      v[4 * w + 3] = x.w;
    }
    tmem_st_32x32b_x8(tdst + (cg * (D / 4) + u * 8) / 2, v);
  }
}

// kv kernel, 32 query columns of one key row: P^T = exp2(S^T*c - LSE*log2e), dS^T = P^T (dP^T - delta),
// LSE / delta per column (shared memory). Columns e outside [lo, hi) are zero (MASK).
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

// q kernel, 32 key columns of one query row: dS = exp2(S*c - LSE*log2e) (dP - delta) with this row's
// LSE / delta. Columns e >= hi are zero (MASK).
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

// DS: also store each (query block, key block) pair's dS^T tile (bf16, 128 keys x 128 queries) for the dQ
// kernel: the element-wise warps write it into one of two shared staging tiles (the 128-byte swizzled
// [64-column chunk][128 rows][128 B] layout), and one thread TMA-stores the tile once all 16 warps have
// arrived; the two tiles alternate, a tile being rewritten only after its previous store has read it
// (bounded mbarrier hand-offs both ways).
template <int D, bool DS>
__global__ void __launch_bounds__(BW_THREADS, 1)
attn_bwd_kv_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDO,
                      const __grid_constant__ CUtensorMap tmLSE, const __grid_constant__ CUtensorMap tmDEL,
                      const __grid_constant__ CUtensorMap tmDS, __nv_bfloat16* __restrict__ dqkv, int B, int T,
                      int nh, int nkv, float scale) {
  using C = KVCfg<D, DS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 599);
    return;
  }
  uint8_t* sK = smem_raw;
  uint8_t* sV = sK + C::TT;
  uint8_t* sQ = sV + C::TT;             // [ST][TT]
  uint8_t* sDO = sQ + C::ST * C::TT;    // [ST][TT]
  float* sLSE = reinterpret_cast<float*>(sDO + C::ST * C::TT);  // [ST][128]
  float* sDEL = sLSE + C::ST * 128;                             // [ST][128]
  uint8_t* sDS = reinterpret_cast<uint8_t*>(sDEL + C::ST * 128);  // [2][128 x 128 bf16] (DS only)
  uint64_t* bar = reinterpret_cast<uint64_t*>(sDS + C::DS_BYTES);
  uint64_t* kv_full = bar;
  uint64_t* qd_full = bar + 1;               // [ST]
  uint64_t* qd_empty = bar + 1 + C::ST;      // [ST]
  uint64_t* s_full = bar + 1 + 2 * C::ST;    // [2] S^T of a buffer computed
  uint64_t* p_full = s_full + 2;             // [2] P^T / dS^T of a buffer written
  uint64_t* dp_full = s_full + 4;            // dP^T computed
  uint64_t* dp_free = s_full + 5;            // dP^T read by the element-wise warps
  uint64_t* mm_done = s_full + 6;
  uint64_t* drain = s_full + 7;
  uint64_t* ds_ready = s_full + 8;           // [2] all element-wise warps wrote a staging tile
  uint64_t* ds_free = s_full + 10;           // [2] a staging tile's previous TMA store has read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (T + 127) / 128;
  // level-major order: every (batch, kv head)'s key block 0 (the most query blocks) is dispatched first,
  // then all key blocks 1, ..., so the last CTAs to start are the shortest (one CTA per SM, not persistent)
  const int nbg = B * nkv;
  const int kb = blockIdx.x / nbg;
  const int bg = blockIdx.x % nbg;
  const int g = bg % nkv, b = bg / nkv;
  const int G = nh / nkv;
  const int nper = nkb - kb;  // causal query blocks kb..nkb-1
  const int iters = G * nper;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < C::ST; ++i) { mbar_init(&qd_full[i], 1); mbar_init(&qd_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], BW_EW_WARPS);
    }
    mbar_init(dp_full, 1);
    mbar_init(dp_free, BW_EW_WARPS);
    mbar_init(mm_done, 1);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ds_ready[i], BW_EW_WARPS);
      mbar_init(&ds_free[i], 1);
    }
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
  const uint32_t tDP = tmem + C::C_DP, tDV = tmem + C::C_DV, tDK = tmem + C::C_DK;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(kv_full, 2 * C::TT);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(sK + c * (128 * 128), &tmQKV, kv_full, (nh + g) * D + 64 * c, kb * 128, b);
        tma_load_3d(sV + c * (128 * 128), &tmQKV, kv_full, (nh + nkv + g) * D + 64 * c, kb * 128, b);
      }
      for (int it = 0; it < iters; ++it) {
        const int hh = it / nper, i = kb + it % nper, h = g * G + hh;
        const int st = it % C::ST;
        if (it >= C::ST &&
            !mbar_wait_bounded(&qd_empty[st], ((it / C::ST) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 500, abort_flag))
          break;
        mbar_arrive_expect_tx(&qd_full[st], 2 * C::TT + 2 * 512);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sQ + st * C::TT + c * (128 * 128), &tmQKV, &qd_full[st], h * D + 64 * c, i * 128, b);
          tma_load_3d(sDO + st * C::TT + c * (128 * 128), &tmDO, &qd_full[st], h * D + 64 * c, i * 128, b);
        }
        tma_load_2d(sLSE + st * 128, &tmLSE, &qd_full[st], i * 128, b * nh + h);
        tma_load_2d(sDEL + st * 128, &tmDEL, &qd_full[st], i * 128, b * nh + h);
        ATTN_TRACE(0, it);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSS = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idKD = umma_idesc_bf16(128, D, 0, 1);
      const uint64_t dK0 = kdesc0(smem_u32(sK)), dV0 = kdesc0(smem_u32(sV));
      const uint64_t dQ0 = kdesc0(smem_u32(sQ)), dDO0 = kdesc0(smem_u32(sDO));
      const uint64_t mQ0 = mndesc0(smem_u32(sQ)), mDO0 = mndesc0(smem_u32(sDO));
      constexpr uint64_t STG = (uint64_t)(C::TT >> 4);  // stage stride in descriptor units
      bool issued = false;
      auto wait_stage = [&](int it) -> bool {
        return mbar_wait_bounded(&qd_full[it % C::ST], (it / C::ST) & 1, DT_ERR_TIMEOUT_FULL, 511, abort_flag);
      };
      // S^T = K Q^T of block `it` into buffer it % NSB
      auto issue_s = [&](int it) {
        const uint64_t q = dQ0 + (uint64_t)(it % C::ST) * STG;
        const uint32_t tS = tmem + (it % C::NSB) * 128;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tS, dK0 + koff(k), q + koff(k), idSS, k > 0 ? 1u : 0u);
        umma_commit(&s_full[it % C::NSB]);
        issued = true;
      };
      // dP^T = V dO^T of block `it`
      auto issue_dp = [&](int it) {
        const uint64_t o = dDO0 + (uint64_t)(it % C::ST) * STG;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16(tDP, dV0 + koff(k), o + koff(k), idSS, k > 0 ? 1u : 0u);
        umma_commit(dp_full);
        ATTN_TRACE(1, it);
      };
      bool ok = mbar_wait_bounded(kv_full, 0, DT_ERR_TIMEOUT_FULL, 510, abort_flag) && wait_stage(0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
      }
      for (int it = 0; it < iters && ok; ++it) {
        const int st = it % C::ST, bb = it % C::NSB;
        const bool more = it + 1 < iters;
        if (more) {
          if (!wait_stage(it + 1)) { ok = false; break; }
          tc_fence_after();
          // a free second buffer: S^T of the next block runs while this block's exponentials do
          if (C::NSB == 2) issue_s(it + 1);
          if (!mbar_wait_bounded(dp_free, it & 1, DT_ERR_TIMEOUT_TMEM, 512, abort_flag)) { ok = false; break; }
          tc_fence_after();
          if (C::NSB == 2) issue_dp(it + 1);
        }
        if (!mbar_wait_bounded(&p_full[bb], (it / C::NSB) & 1, DT_ERR_TIMEOUT_FULL, 513, abort_flag)) { ok = false; break; }
        ATTN_TRACE(2, it);
        tc_fence_after();
        const uint32_t tS = tmem + bb * 128;
        const uint64_t mq = mQ0 + (uint64_t)st * STG, mo = mDO0 + (uint64_t)st * STG;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          umma_bf16_ts(tDV, pcol(tS, 0, k), mo + mnoff(k), idKD, (it > 0 || k > 0) ? 1u : 0u);
          umma_bf16_ts(tDK, pcol(tS, 1, k), mq + mnoff(k), idKD, (it > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&qd_empty[st]);
        ATTN_TRACE(7, it);
        if (C::NSB == 1 && more) {  // the single buffer is free once dV / dK of this block are issued
          issue_s(it + 1);
          issue_dp(it + 1);
        }
      }
      if (ok) umma_commit(mm_done);
      if (!ok && issued) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    // ───── element-wise warps: thread = key row r, query columns [cg*32, cg*32+32) of the block ─────
    const int ew = warp - 2, quad = warp & 3, cg = ew >> 2;
    const int r = quad * 32 + lane;
    const int key = kb * 128 + r;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sl2 = scale * LOG2E_F;
    const bool edge_k = (kb + 1) * 128 > T;
    WarpWait wwait{abort_flag, lane};
    bool ok = true;
    for (int it = 0; it < iters && ok; ++it) {
      const int i = kb + it % nper;
      const int st = it % C::ST, bb = it % C::NSB;
      const uint32_t tS = tmem + bb * 128 + lane_off + cg * 32;
      uint32_t pk[16], dk[16];
      {
        uint32_t sv[32], dv[32];
        if (!wwait(&s_full[bb], (it / C::NSB) & 1, 520)) { ok = false; break; }
        tc_fence_after();
        tmem_ld_32x32b_x32(tS, sv);
        if (!wwait(dp_full, it & 1, 521)) { ok = false; break; }
        if (warp == 2 && lane == 0) ATTN_TRACE(3, it);
        tc_fence_after();
        tmem_ld_32x32b_x32(tDP + lane_off + cg * 32, dv);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(dp_free, lane);
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
      if constexpr (DS) {
        // dS^T of this (query block i, key block kb) pair: row = key r, query columns cg*32..+32
        const int db = it & 1;
        if (it >= 2 && !wwait(&ds_free[db], ((it >> 1) - 1) & 1, 530)) { ok = false; break; }
        uint8_t* tile = sDS + db * (128 * 128 * 2) + (cg >> 1) * (128 * 128) + r * 128;
#pragma unroll
        for (int v = 0; v < 4; ++v)
          *reinterpret_cast<uint4*>(tile + ((((cg & 1) * 4 + v) ^ (r & 7)) << 4)) =
              make_uint4(dk[4 * v], dk[4 * v + 1], dk[4 * v + 2], dk[4 * v + 3]);
        fence_proxy_async_smem();
        warp_arrive(&ds_ready[db], lane);
        if (warp == 2 && lane == 0) {
          if (!mbar_wait_bounded(&ds_ready[db], (it >> 1) & 1, DT_ERR_TIMEOUT_FULL, 531, abort_flag)) {
            ok = false;
          } else {
            if (it >= 1) {  // the other tile's store (issued one block ago) has read it: free for block it+1
              bulk_wait_read0();
              mbar_arrive(&ds_free[db ^ 1]);
            }
            const int hh = it / nper, h = g * G + hh;
            const long long pair =
                ((long long)b * nh + h) * ((long long)nkb * (nkb + 1) / 2) + (long long)i * (i + 1) / 2 + kb;
            uint8_t* t0 = sDS + db * (128 * 128 * 2);
            tma_store_2d(&tmDS, t0, 0, (int)(pair * 128));
            tma_store_2d(&tmDS, t0 + 128 * 128, 64, (int)(pair * 128));
            bulk_commit();
          }
        }
        __syncwarp();
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
      tmem_st_32x32b_x16(tS, pk);
      tmem_st_32x32b_x16(tS + 16, dk);
      tmem_st_wait();
      tc_fence_before();
      if (warp == 2 && lane == 0) ATTN_TRACE(4, it);
      warp_arrive(&p_full[bb], lane);
    }
    // epilogue: dK (scaled) and dV rows of this key block, D/4 columns per thread
    if (ok && wwait(mm_done, 0, 522)) {
      tc_fence_after();
      const long long W = (long long)(nh + 2 * nkv) * D;
      __nv_bfloat16* krow = dqkv + ((long long)b * T + key) * W + (nh + g) * D + cg * (D / 4);
      __nv_bfloat16* vrow = dqkv + ((long long)b * T + key) * W + (nh + nkv + g) * D + cg * (D / 4);
      tmem_row_to_bf16(tDK + lane_off + cg * (D / 4), D / 4, scale, key < T, krow);
      tmem_row_to_bf16(tDV + lane_off + cg * (D / 4), D / 4, 1.f, key < T, vrow);
    }
    if (DS && warp == 2 && lane == 0) bulk_wait0();  // the dS^T stores have completed
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
  uint8_t* sDO = sQ + C::TT;
  uint8_t* sK = sDO + C::TT;          // [ST][TT]
  uint8_t* sV = sK + C::ST * C::TT;   // [ST][TT]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sV + C::ST * C::TT);
  uint64_t* q_full = bar;
  uint64_t* kv_full = bar + 1;               // [ST]
  uint64_t* kv_empty = bar + 1 + C::ST;      // [ST]
  uint64_t* s_full = bar + 1 + 2 * C::ST;    // [2]
  uint64_t* p_full = s_full + 2;             // [2]
  uint64_t* dp_full = s_full + 4;
  uint64_t* dp_free = s_full + 5;
  uint64_t* qt_full = s_full + 6;            // Q / dO copied into TMEM
  uint64_t* mm_done = s_full + 7;
  uint64_t* drain = s_full + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (T + 127) / 128;
  // level-major order: the last query block (the most key blocks) of every (batch, head) first
  const int nbh = B * nh;
  const int qb = nqb - 1 - blockIdx.x / nbh;
  const int bh = blockIdx.x % nbh;
  const int h = bh % nh, b = bh / nh;
  const int g = h / (nh / nkv);
  const int njb = qb + 1;  // causal key blocks 0..qb

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::ST; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], BW_EW_WARPS);
    }
    mbar_init(dp_full, 1);
    mbar_init(dp_free, BW_EW_WARPS);
    mbar_init(qt_full, BW_EW_WARPS);
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
  const uint32_t tDP = tmem + C::C_DP, tDQ = tmem + C::C_DQ, tQ = tmem + C::C_Q, tDO = tmem + C::C_DO;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(q_full, 2 * C::TT);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(sQ + c * (128 * 128), &tmQKV, q_full, h * D + 64 * c, qb * 128, b);
        tma_load_3d(sDO + c * (128 * 128), &tmDO, q_full, h * D + 64 * c, qb * 128, b);
      }
      for (int j = 0; j < njb; ++j) {
        const int st = j % C::ST;
        if (j >= C::ST &&
            !mbar_wait_bounded(&kv_empty[st], ((j / C::ST) & 1) ^ 1, DT_ERR_TIMEOUT_EMPTY, 600, abort_flag))
          break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::TT);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma_load_3d(sK + st * C::TT + c * (128 * 128), &tmQKV, &kv_full[st], (nh + g) * D + 64 * c, j * 128, b);
          tma_load_3d(sV + st * C::TT + c * (128 * 128), &tmQKV, &kv_full[st], (nh + nkv + g) * D + 64 * c, j * 128, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idSS = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idQD = umma_idesc_bf16(128, D, 0, 1);
      const uint64_t dK0 = kdesc0(smem_u32(sK)), dV0 = kdesc0(smem_u32(sV)), mK0 = mndesc0(smem_u32(sK));
      constexpr uint64_t STG = (uint64_t)(C::TT >> 4);
      bool issued = false;
      auto wait_stage = [&](int j) -> bool {
        return mbar_wait_bounded(&kv_full[j % C::ST], (j / C::ST) & 1, DT_ERR_TIMEOUT_FULL, 611, abort_flag);
      };
      auto issue_s = [&](int j) {  // S = Q K^T of key block j into buffer j % NSB
        const uint64_t kk = dK0 + (uint64_t)(j % C::ST) * STG;
        const uint32_t tS = tmem + (j % C::NSB) * 128;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16_ts(tS, tQ + k * 8, kk + koff(k), idSS, k > 0 ? 1u : 0u);
        umma_commit(&s_full[j % C::NSB]);
        issued = true;
      };
      auto issue_dp = [&](int j) {  // dP = dO V^T of key block j
        const uint64_t vv = dV0 + (uint64_t)(j % C::ST) * STG;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) umma_bf16_ts(tDP, tDO + k * 8, vv + koff(k), idSS, k > 0 ? 1u : 0u);
        umma_commit(dp_full);
      };
      bool ok = mbar_wait_bounded(qt_full, 0, DT_ERR_TIMEOUT_FULL, 610, abort_flag) && wait_stage(0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        issue_dp(0);
      }
      for (int j = 0; j < njb && ok; ++j) {
        const int st = j % C::ST, bb = j % C::NSB;
        const bool more = j + 1 < njb;
        if (more) {
          if (!wait_stage(j + 1)) { ok = false; break; }
          tc_fence_after();
          if (C::NSB == 2) issue_s(j + 1);
          if (!mbar_wait_bounded(dp_free, j & 1, DT_ERR_TIMEOUT_TMEM, 612, abort_flag)) { ok = false; break; }
          tc_fence_after();
          if (C::NSB == 2) issue_dp(j + 1);
        }
        if (!mbar_wait_bounded(&p_full[bb], (j / C::NSB) & 1, DT_ERR_TIMEOUT_FULL, 613, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tS = tmem + bb * 128;
        const uint64_t mk = mK0 + (uint64_t)st * STG;
#pragma unroll
        for (int k = 0; k < 8; ++k) umma_bf16_ts(tDQ, pcol(tS, 0, k), mk + mnoff(k), idQD, (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(&kv_empty[st]);
        if (C::NSB == 1 && more) {
          issue_s(j + 1);
          issue_dp(j + 1);
        }
      }
      if (ok) umma_commit(mm_done);
      if (!ok && issued) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    // ───── element-wise warps: thread = query row r, key columns [cg*32, cg*32+32) of the block ─────
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
    bool ok = wwait(q_full, 0, 623);
    if (ok) {
      tile_row_to_tmem<D>(sQ, r, cg, tQ + lane_off);
      tile_row_to_tmem<D>(sDO, r, cg, tDO + lane_off);
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(qt_full, lane);
    }
    for (int j = 0; j < njb && ok; ++j) {
      const int bb = j % C::NSB;
      const uint32_t tS = tmem + bb * 128 + lane_off + cg * 32;
      uint32_t dk[16];
      {
        uint32_t sv[32], dv[32];
        if (!wwait(&s_full[bb], (j / C::NSB) & 1, 620)) { ok = false; break; }
        tc_fence_after();
        tmem_ld_32x32b_x32(tS, sv);
        if (!wwait(dp_full, j & 1, 621)) { ok = false; break; }
        tc_fence_after();
        tmem_ld_32x32b_x32(tDP + lane_off + cg * 32, dv);
        tmem_ld_wait();
        tc_fence_before();
        warp_arrive(dp_free, lane);
        if (j == qb || edge_q || (j + 1) * 128 > T) {
          const int kbase = j * 128 + cg * 32;
          const int hi = q < T ? min(q - kbase + 1, T - kbase) : 0;  // valid columns: e < hi
          q_block_math<true>(sv, dv, sl2, nlse2, dlt, hi, dk);
        } else {
          q_block_math<false>(sv, dv, sl2, nlse2, dlt, 32, dk);
        }
      }
      tmem_st_32x32b_x16(tS, dk);
      tmem_st_wait();
      tc_fence_before();
      warp_arrive(&p_full[bb], lane);
    }
    if (ok && wwait(mm_done, 0, 622)) {
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

// dQ from the stored dS^T tiles: dQ[q, :] = scale * sum over causal key blocks j of dS[q, keys of j] K[keys of j, :].
// A batched GEMM with no exponentials (the kv kernel formed dS once): persistent CTAs over (batch, head,
// query block) tiles, heaviest first; warp 0 streams the dS^T tile (as the MN-major A operand) and the K
// tile (MN-major B) of each pair through a TMA ring, warp 1 issues tcgen05.mma into one of two TMEM
// accumulators, warps 2..5 scale and store the finished dQ rows while the next tile accumulates.
template <int D>
struct DQCfg {
  static constexpr int A_BYTES = 128 * 128 * 2;   // dS^T tile
  static constexpr int B_BYTES = 128 * D * 2;     // K tile
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int ST = (232448 - 1024 - 256) / STAGE < 4 ? (232448 - 1024 - 256) / STAGE : 4;
  static constexpr int SMEM = ST * STAGE + 256;
  static constexpr int TMEM_COLS = 2 * D;
};
constexpr int DQ_THREADS = 192;

template <int D>
__global__ void __launch_bounds__(DQ_THREADS, 1)
attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmDS,
                      __nv_bfloat16* __restrict__ dqkv, int B, int T, int nh, int nkv, float scale) {
  using C = DQCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {
    if (threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 699);
    return;
  }
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem_raw + C::ST * C::STAGE);
  uint64_t* full = bar;                 // [ST]
  uint64_t* empty = bar + C::ST;        // [ST]
  uint64_t* tfull = bar + 2 * C::ST;    // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (T + 127) / 128;
  const int ntiles = B * nh * nqb;
  const long long P = (long long)nqb * (nqb + 1) / 2;  // stored pairs per (batch, head)
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::ST; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 128); }
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
  auto tile_of = [&](int t, int& b, int& h, int& qb) {
    const int bh_count = B * nh;
    qb = nqb - 1 - t / bh_count;
    const int bh = t % bh_count;
    h = bh % nh;
    b = bh / nh;
  };
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQKV);
      tma_prefetch_desc(&tmDS);
      int stage = 0, phase = 0, issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        int b, h, qb;
        tile_of(t, b, h, qb);
        const int g = h / (nh / nkv);
        const long long pair0 = ((long long)b * nh + h) * P + (long long)qb * (qb + 1) / 2;
        for (int j = 0; j <= qb; ++j) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, DT_ERR_TIMEOUT_EMPTY, 640, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], C::STAGE);
          uint8_t* a = smem_raw + stage * C::STAGE;
          uint8_t* kb = a + C::A_BYTES;
          tma_load_2d(a, &tmDS, &full[stage], 0, (int)((pair0 + j) * 128));
          tma_load_2d(a + 128 * 128, &tmDS, &full[stage], 64, (int)((pair0 + j) * 128));
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_3d(kb + c * (128 * 128), &tmQKV, &full[stage], (nh + g) * D + 64 * c, j * 128, b);
          ++issued;
          if (++stage == C::ST) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        uint64_t t0 = dt_globaltimer();
        for (int k = (issued > C::ST ? issued - C::ST : 0); k < issued; ++k)
          while (!mbar_try_wait(&full[k % C::ST], (k / C::ST) & 1) && dt_globaltimer() - t0 < 20000000ull) {}
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, D, 1, 1);
      int stage = 0, phase = 0, local = 0;
      bool ok = true, issued_any = false;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++local) {
        int b, h, qb;
        tile_of(t, b, h, qb);
        const int acc = local & 1;
        if (!mbar_wait_bounded(&tempty[acc], ((local >> 1) & 1) ^ 1, DT_ERR_TIMEOUT_TMEM, 641, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tacc = tmem + acc * D;
        for (int j = 0; j <= qb; ++j) {
          if (!mbar_wait_bounded(&full[stage], phase, DT_ERR_TIMEOUT_FULL, 642, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = smem_u32(smem_raw + stage * C::STAGE);
          const uint64_t mA = mndesc0(a), mB = umma_smem_desc_sw128(a + C::A_BYTES, 128 * 128, 1024);
#pragma unroll
          for (int k = 0; k < 8; ++k) umma_bf16(tacc, mA + mnoff(k), mB + mnoff(k), idesc, (j > 0 || k > 0) ? 1u : 0u);
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == C::ST) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    }
  } else {
    const int quad = warp & 3;
    const long long W = (long long)(nh + 2 * nkv) * D;
    int local = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++local) {
      int b, h, qb;
      tile_of(t, b, h, qb);
      const int acc = local & 1;
      if (!mbar_wait_bounded(&tfull[acc], (local >> 1) & 1, DT_ERR_TIMEOUT_TMEM, 643, abort_flag)) break;
      tc_fence_after();
      const int q = qb * 128 + quad * 32 + lane;
      __nv_bfloat16* qrow = dqkv + ((long long)b * T + q) * W + h * D;
      tmem_row_to_bf16(tmem + ((uint32_t)(quad * 32) << 16) + acc * D, D, scale, q < T, qrow);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
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
                  int nh, int nkv, float scale, cudaStream_t st, void* ds_buf = nullptr) {
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
    DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_kv_tc_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     KVCfg<D>::SMEM));
    if (D == 64)
      DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_kv_tc_kernel<D, D == 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       KVCfg<D, D == 64>::SMEM));
    DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_q_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, QCfg<D>::SMEM));
    DT_CUDA_RET(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, DQCfg<D>::SMEM));
    set = true;
  }
  const int nb = (T + 127) / 128;
  auto dq = reinterpret_cast<__nv_bfloat16*>(dqkv);
  if (ds_buf && D == 64) {
    // dQ from the stored dS^T tiles: no second pass over the exponentials
    const long long rows = (long long)B * nh * ((long long)nb * (nb + 1) / 2) * 128;
    if (rows > 0x7fffffffLL) return -12;
    CUtensorMap mds;
    cuuint64_t dims[2] = {128, (cuuint64_t)rows};
    cuuint64_t strides[1] = {256};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    if (g_enc(&mds, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ds_buf, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
        CUDA_SUCCESS)
      return -3;
    attn_bwd_kv_tc_kernel<D, D == 64><<<B * nkv * nb, BW_THREADS, KVCfg<D, D == 64>::SMEM, st>>>(
        mq, mdo, ml, md, mds, dq, B, T, nh, nkv, scale);
    DT_CUDA_RET(cudaGetLastError());
    static int sms = 0;
    if (!sms) {
      int dev = 0;
      DT_CUDA_RET(cudaGetDevice(&dev));
      DT_CUDA_RET(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    }
    const int tiles = B * nh * nb;
    attn_bwd_dq_tc_kernel<D><<<tiles < sms ? tiles : sms, DQ_THREADS, DQCfg<D>::SMEM, st>>>(mq, mds, dq, B, T, nh, nkv,
                                                                                          scale);
    return (int)cudaGetLastError();
  }
  attn_bwd_kv_tc_kernel<D, false><<<B * nkv * nb, BW_THREADS, KVCfg<D>::SMEM, st>>>(mq, mdo, ml, md, md, dq, B, T, nh,
                                                                                   nkv, scale);
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

// Bytes of the dS^T buffer dt_attn_bwd_tc_ds needs: one 128 x 128 bf16 tile per causal (query block, key block)
// pair of every (batch, head).
DT_API long long dt_attn_ds_bytes(int B, int T, int nh) {
  const long long nb = (T + 127) / 128;
  return (long long)B * nh * (nb * (nb + 1) / 2) * 128 * 128 * 2;
}

// tcgen05 backward whose kv kernel also stores dS^T (bf16) into ds_buf (dt_attn_ds_bytes, 16-byte aligned), from
// which a GEMM-like kernel forms dQ without recomputing S and P.
// (Head dim 128 keeps the recomputing dQ kernel: its key-block kernel has no room for the staging tiles.)
DT_API int dt_attn_bwd_tc_ds(const void* qkv, const void* dout, const float* lse, const float* delta, void* dqkv,
                             void* ds_buf, int B, int T, int nh, int nkv, int D, float scale, cudaStream_t st) {
  if (nh % nkv || !ds_buf || (reinterpret_cast<uintptr_t>(ds_buf) & 15)) return -10;
  if (D == 64) return bwd_tc_launch<64>(qkv, dout, lse, delta, dqkv, B, T, nh, nkv, scale, st, ds_buf);
  if (D == 128) return bwd_tc_launch<128>(qkv, dout, lse, delta, dqkv, B, T, nh, nkv, scale, st, ds_buf);
  return -11;
}
