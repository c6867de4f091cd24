// Persistent tcgen05 GEMM for sm_100a:   C[M,N] (op)= alpha * sum_k A[m,k] * B[n,k]
//
// * Operands are bf16 in global memory, staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, no
//   cluster multicast) into a STAGES-deep shared-memory ring; each operand may be K-major
//   (k contiguous) or MN-major (m / n contiguous), which covers forward (X W^T), data-gradient
//   (dY W) and weight-gradient (dY^T X) products without any transpose pass.
// * One elected thread of warp 1 issues tcgen05.mma (M=128, N=BN, K=16, fp32 accumulate) into one
//   of two TMEM accumulators; tcgen05.commit releases shared-memory stages and hands finished
//   accumulators to the epilogue, so the epilogue of tile i overlaps the main loop of tile i+1.
// * Warps 2..9 (two per TMEM lane quadrant, each half of the tile's columns) drain TMEM with tcgen05.ld
//   (32 lanes x 32 columns per load) into swizzled shared staging boxes and write them with a TMA store
//   (bf16 / fp32) or a TMA reduce-add (fp32 accumulation, used for split-K and gradient accumulation), so
//   global writes are full-line and asynchronous.
// * Tiles are visited by a persistent grid (one CTA per SM) in grouped order for L2 reuse.
// * The plain GEMM's 256-wide tiles run on CTA pairs (clusters of two SMs, tcgen05 cta_group::2): a pair computes a
//   256 x 256 tile with M = 256 MMAs issued by its even CTA; each CTA stages its own 128 rows of A and
//   128 of the 256 B rows, so per output it reads 3/4 of the operand bytes of a single-CTA 128 x 256
//   tile. Operand loads of both CTAs complete on the even CTA's barriers; the MMA commits arrive on both
//   CTAs' barriers; both CTAs' epilogues hand TMEM back to the even CTA. No load uses multicast.
// * Fused SwiGLU (reference model.rs:292-296, h = silu(x Wg^T) * (x Wu^T)):
//     forward (MODE 1): one 256-wide tile holds 128 gate columns and the 128 matching up columns (the B
//       stage is filled from the gate rows and the up rows of the [2F, K] weight by two TMA loads); the
//       epilogue stores gate and up (bf16, kept for the backward) and h = silu(g) * u from the fp32
//       accumulators, so no separate activation pass reads the [M, 2F] product back;
//     backward (MODE 2): the down-projection data gradient dh = dY Wd is never stored - the epilogue
//       reads the saved gate / up values of its rows and writes dgate = dh * u * silu'(g) and
//       dup = dh * silu(g) straight into the [M, 2F] gradient the gate/up GEMMs consume.
// * LM head with softmax statistics (MODE 4, reference model.rs:323-339 and 804-811): besides the bf16
//   logits, the epilogue keeps, per row and half tile, the running max and sum of exp of the fp32
//   accumulators and the fp32 logit of the row's target token, so the cross-entropy's log-sum-exp and
//   loss come from fp32 values and need no pass over the logits.
// * Fused QKV bias + rotary embedding (MODE 3, reference model.rs:193-201 and 66-122): the QKV GEMM's
//   epilogue adds the bias and applies the rotate-half rotation of every q / k head (position = row mod
//   T, fp32 cos/sin tables [T, d/2]) before the single bf16 store; v heads get the bias only.
// Every mbarrier wait is bounded (common.cuh); on timeout the CTA drains its in-flight TMA loads and
// MMAs, frees TMEM and returns with dt_error_word set.
#include "common.cuh"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>
#include <cstdlib>

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int EPI_WARPS = 8;                        // two per TMEM lane quadrant
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;    // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int GROUP_M = 16;

enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_F32_ATOMIC = 2 };

struct GemmArgs {
  int M, N, K;
  // fused SwiGLU backward: the saved [M, 2F] gate|up product (row stride ld_gu), F = N
  const __nv_bfloat16* gu;
  long long ld_gu;
  // fused QKV bias + RoPE: tables [T, hd/2], bias [N] (nullable), columns [0, rot_cols) are rotated heads
  const float* cosT;
  const float* sinT;
  const float* bias;
  int T, hd, rot_cols;
  // logits + softmax statistics (MODE 4): per (row, tile column half) max and sum of exp of the fp32
  // logits, and the fp32 logit of the row's target token (ids[b*S + t + 1], global row r0 + row)
  float2* lse_part;
  float* tgt_logit;
  const int* ids;
  int S;
  long long r0;
  int num_kb;
  int split_k, kb_per_split;
  int tiles_m, tiles_n;
  int epi;
  float alpha;
  void* C;
  long long ldc;
  // Tensor-parallel partial-sum exchange (bf16 epilogue only): every output box is also TMA-stored
  // into the peer GPU's receive buffer (tmCp, over NVLink); once all CTAs' stores have completed, the
  // last CTA adds 1 to the peer's arrival counter with a system-scope release.
  int peer;
  unsigned* peer_arrivals;  // on the peer GPU
  unsigned* done_ctas;      // local scratch counter, returns to 0 after every launch
};

template <int BN, int MODE = 0, bool PAIR = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // a CTA of a pair holds half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int TMEM_ALLOC = TMEM_COLS <= 256 ? 256 : 512;  // allocations are powers of two
  // columns of a tile drained by the first epilogue warp of a lane quadrant (the second takes the rest)
  static constexpr int COL_SPLIT = BN == 192 ? 128 : BN / 2;
  static_assert(COL_SPLIT % 64 == 0 && (BN - COL_SPLIT) % 64 == 0, "epilogue boxes are 64 bf16 / 32 fp32 wide");
  static constexpr int BOXES = (MODE == 0 || MODE == 4) ? 1 : 2;  // 4 KB staging boxes per epilogue warp
  static constexpr int EPI_BYTES = EPI_WARPS * BOXES * 4096;
  static constexpr int FIXED = EPI_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
  // as many operand stages as fit next to the staging boxes (at most 6)
  static constexpr int STAGES = (232448 - FIXED) / STAGE_BYTES < 6 ? (232448 - FIXED) / STAGE_BYTES : 6;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + FIXED;
  static_assert(STAGES >= 3, "operand ring");
};

__device__ __forceinline__ void tile_coords(int tile, int tiles_m, int tiles_n, int& mb, int& nb) {
  int group = GROUP_M * tiles_n;
  int g = tile / group;
  int first_m = g * GROUP_M;
  int gm = min(tiles_m - first_m, GROUP_M);
  int within = tile - g * group;
  mb = first_m + within % gm;
  nb = within / gm;
}

// logistic function with the hardware exponential and reciprocal (the activations are rounded to bf16)
__device__ __forceinline__ float sigmoid_f(float x) { return __frcp_rn(1.f + __expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_f(x); }

// 16-byte chunk `ch` (8 bf16) of row `lane` of a 32-row x 128-byte staging box in the TMA 128-byte
// swizzle layout (chunk k of row r stored at k ^ (r & 7)), so the 32 lanes' stores spread over all banks
__device__ __forceinline__ void box_put(uint8_t* box, int lane, int ch, uint4 v) {
  *reinterpret_cast<uint4*>(box + lane * 128 + ((ch ^ (lane & 7)) * 16)) = v;
}

// PAIR: the kernel runs as clusters of two CTAs on two SMs, each pair computing 256 x BN tiles with
// cta_group::2 MMAs (M = 256): each CTA loads its 128 rows of A and BN/2 rows (columns of the product)
// of B, so a CTA reads (128 + BN/2) x K operand elements per 128 x BN outputs instead of (128 + BN) x K.
template <int BN, int A_MN, int B_MN, int MODE, bool PAIR = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmCp,
               const __grid_constant__ CUtensorMap tmB2, const __grid_constant__ CUtensorMap tmC2,
               const __grid_constant__ CUtensorMap tmC3, GemmArgs args) {
  static_assert(MODE != 1 || (BN == 256 && !A_MN && !B_MN), "fused SwiGLU forward: 128 gate + 128 up columns");
  static_assert(!PAIR || ((BN == 128 || BN == 256) && MODE != 2), "CTA pairs: 128- or 256-wide tiles, not MODE 2");
  using C = Cfg<BN, MODE, PAIR>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sEpi = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + C::EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* tfull = bars + 2 * C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* gbar = drain + 1;  // [EPI_WARPS] per-warp operand loads of the SwiGLU backward epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbar + EPI_WARPS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], (PAIR ? 2 : 1) * 32 * EPI_WARPS);
    }
    mbar_init(drain, 1);
    for (int w = 0; w < EPI_WARPS; ++w) mbar_init(&gbar[w], 1);
    *abort_flag = 0;
    *consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
    if (MODE == 1 || MODE == 2) {
      tma_prefetch_desc(&tmC2);
      tma_prefetch_desc(&tmB2);
      tma_prefetch_desc(&tmC3);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_ALLOC);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_ALLOC);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  // a pair's CTAs signal each other's barriers: both must have initialised theirs first
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int crank = PAIR ? (int)cluster_ctarank() : 0;
  // a pair's MMAs write both CTAs' TMEM at the even CTA's address: both allocations must agree, else
  // nothing runs and the error word is set
  bool pair_ok = true;
  if constexpr (PAIR) {
    pair_ok = ld_shared_cluster_u32(mapa_shared(smem_u32(tmem_slot), crank ^ 1)) == tmem_base;
    if (!pair_ok && threadIdx.x == 0) dt_set_error(DT_ERR_BAD_ARG, 150);
  }

  const int total_units = pair_ok ? args.tiles_m * args.tiles_n * args.split_k : 0;
  // persistent walk: a CTA (or a pair of CTAs) takes units first, first + step, ...
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int TM = PAIR ? 2 * BM : BM;  // rows of a tile (a pair's tile spans both CTAs)
  const int mrow = crank * BM;        // this CTA's rows within the tile
  // barriers of the even CTA, where a pair's operand loads complete and its epilogues hand TMEM back
  auto lead = [&](uint64_t* b) -> uint32_t { return PAIR ? mapa_shared(smem_u32(b), 0) : smem_u32(b); };
  // an epilogue thread has read its TMEM columns of accumulator `acc`
  auto arrive_tempty = [&](int acc) {
    if constexpr (PAIR) mbar_arrive_remote(lead(&tempty[acc]));
    else mbar_arrive(&tempty[acc]);
  };

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      int issued = 0;
      bool ok = true;
      for (int unit = unit0; unit < total_units && ok; unit += ustep) {
        int s = unit % args.split_k, tile = unit / args.split_k;
        int mb, nb;
        tile_coords(tile, args.tiles_m, args.tiles_n, mb, nb);
        int m0 = mb * TM + mrow, n0 = nb * (MODE == 1 ? BN / 2 : BN);
        int kb0 = s * args.kb_per_split, kb1 = min(kb0 + args.kb_per_split, args.num_kb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, DT_ERR_TIMEOUT_EMPTY, 100, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          if constexpr (PAIR) {
            // both CTAs' loads complete on the even CTA's barrier, which expects the pair's bytes
            const uint32_t fb = lead(&full[stage]);
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            if (A_MN) {
#pragma unroll
              for (int j = 0; j < BM / 64; ++j) tma_load_2d_pair(a_dst + j * (64 * BK * 2), &tmA, fb, m0 + 64 * j, kb * BK);
            } else {
              tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, m0);
            }
            if (MODE == 1) {
              // the even CTA holds the tile's 128 gate rows of B, the odd one the matching up rows
              tma_load_2d_pair(b_dst, crank ? &tmB2 : &tmB, fb, kb * BK, n0);
            } else if (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tma_load_2d_pair(b_dst + j * (64 * BK * 2), &tmB, fb, n0 + crank * (BN / 2) + 64 * j, kb * BK);
            } else {
              tma_load_2d_pair(b_dst, &tmB, fb, kb * BK, n0 + crank * (BN / 2));
            }
            ++issued;
            if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * (64 * BK * 2), &tmA, &full[stage], m0 + 64 * j, kb * BK);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, m0);
          }
          if (MODE == 1) {
            // gate rows [n0, n0+128) then the matching up rows: two 128-row boxes, the same swizzled
            // layout as one 256-row box
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, n0);
            tma_load_2d(b_dst + (BN / 2) * BK * 2, &tmB2, &full[stage], kb * BK, n0);
          } else if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * (64 * BK * 2), &tmB, &full[stage], n0 + 64 * j, kb * BK);
          } else {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, n0);
          }
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag && crank == 0) {
        // Drain: wait (bounded) for every issued-but-unconsumed stage so no TMA write lands after exit (a
        // pair's loads all complete on the even CTA's barriers; the final cluster barrier holds the odd
        // CTA until then).
        for (int i = *consumed; i < issued; ++i) {
          uint64_t t0 = dt_globaltimer();
          while (!mbar_try_wait(&full[i % C::STAGES], (i / C::STAGES) & 1)) {
            if (dt_globaltimer() - t0 > 20000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ───────────── MMA issuer (the even CTA of a pair issues for both) ─────────────
    if (lane == 0 && crank == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(PAIR ? 2 * BM : BM, BN, A_MN, B_MN);
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      // commit to a barrier of this CTA and, for a pair, to the same barrier of the odd CTA
      auto commit_both = [&](uint64_t* b) {
        if constexpr (PAIR) {
          umma_commit_pair(smem_u32(b));
          umma_commit_pair(mapa_shared(smem_u32(b), 1));
        } else {
          umma_commit(b);
        }
      };
      for (int unit = unit0; unit < total_units && ok; unit += ustep, ++local) {
        int s = unit % args.split_k;
        int kb0 = s * args.kb_per_split, kb1 = min(kb0 + args.kb_per_split, args.num_kb);
        int acc = local & 1;
        uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, DT_ERR_TIMEOUT_TMEM, 200, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, DT_ERR_TIMEOUT_FULL, 201, abort_flag)) { ok = false; break; }
          *consumed = *consumed + 1;
          tc_fence_after();
          uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad = A_MN ? umma_smem_desc_sw128(a_addr + k * 2048, 64 * BK * 2, 1024)
                               : umma_smem_desc_sw128(a_addr + k * 32, 16, 1024);
            uint64_t bd = B_MN ? umma_smem_desc_sw128(b_addr + k * 2048, 64 * BK * 2, 1024)
                               : umma_smem_desc_sw128(b_addr + k * 32, 16, 1024);
            if constexpr (PAIR) umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
            else umma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          issued_any = true;
          commit_both(&empty[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        commit_both(&tfull[acc]);
      }
      if (!ok && issued_any) {
        // Make sure every issued MMA has retired before TMEM is released.
        if constexpr (PAIR) umma_commit_pair(smem_u32(drain));
        else umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) {
          if (dt_globaltimer() - t0 > 20000000ull) break;
        }
      }
    }
  } else {
    // ───────────── Epilogue: warps 2..9 ─────────────
    // Two warps per TMEM lane quadrant (warp w may read lanes 32*(w%4)..+31), each draining half of the
    // tile's columns: TMEM -> registers (tcgen05.ld) -> swizzled 4 KB shared staging box(es) -> TMA store
    // or TMA reduce-add (fp32 accumulation); the tensor maps clip the M / N tails.
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int hsel = ew >> 2;  // which half of the tile's columns this warp drains
    uint8_t* stage = sEpi + ew * (C::BOXES * 4096);
    int local = 0;
    bool pending = false;
    if constexpr (MODE == 2) {
      // SwiGLU backward: this warp's 32 rows x 64 columns of the saved gate / up values arrive by TMA in
      // its two staging boxes (issued one tile ahead), are overwritten in place with dgate / dup and
      // stored from there.
      uint64_t* gb = &gbar[ew];
      auto prefetch = [&](int u) {
        int mb, nb;
        tile_coords(u / args.split_k, args.tiles_m, args.tiles_n, mb, nb);
        if (lane == 0) {
          mbar_arrive_expect_tx(gb, 8192);
          tma_load_2d(stage, &tmB2, gb, nb * BN + hsel * 64, mb * TM + mrow + quad * 32);
          tma_load_2d(stage + 4096, &tmC3, gb, nb * BN + hsel * 64, mb * TM + mrow + quad * 32);
        }
        __syncwarp();
      };
      bool inflight = false;
      if (unit0 < total_units) {
        prefetch(unit0);
        inflight = true;
      }
      for (int unit = unit0; unit < total_units; unit += ustep, ++local) {
        int mb, nb;
        tile_coords(unit / args.split_k, args.tiles_m, args.tiles_n, mb, nb);
        const int acc = local & 1;
        if (!mbar_wait_bounded(&tfull[acc], (local >> 1) & 1, DT_ERR_TIMEOUT_TMEM, 300, abort_flag)) break;
        if (!mbar_wait_bounded(gb, local & 1, DT_ERR_TIMEOUT_FULL, 301, abort_flag)) break;
        inflight = false;
        tc_fence_after();
        const int row0 = mb * TM + mrow + quad * 32;
        const int gcol = nb * BN + hsel * 64;
        const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + hsel * 64;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t d[32];
          tmem_ld_32x32b_x32(t_row + 32 * half, d);
          tmem_ld_wait();
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            const int off = lane * 128 + (((half * 4 + ch) ^ (lane & 7)) * 16);
            uint4* pg = reinterpret_cast<uint4*>(stage + off);
            uint4* pu = reinterpret_cast<uint4*>(stage + 4096 + off);
            const uint4 gv = *pg, uv = *pu;
            const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
            const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
            uint32_t og[4], ou[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 a = unpack_bf16(gw[e]), b = unpack_bf16(uw[e]);
              const float d0 = __uint_as_float(d[ch * 8 + 2 * e]), d1 = __uint_as_float(d[ch * 8 + 2 * e + 1]);
              const float s0 = sigmoid_f(a.x), s1 = sigmoid_f(a.y);
              const float ds0 = s0 * (1.f + a.x * (1.f - s0)), ds1 = s1 * (1.f + a.y * (1.f - s1));
              og[e] = pack_bf16(d0 * b.x * ds0, d1 * b.y * ds1);
              ou[e] = pack_bf16(d0 * a.x * s0, d1 * a.y * s1);
            }
            *pg = make_uint4(og[0], og[1], og[2], og[3]);
            *pu = make_uint4(ou[0], ou[1], ou[2], ou[3]);
          }
        }
        tc_fence_before();
        arrive_tempty(acc);  // this warp's TMEM columns are read
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (gcol < args.N && row0 < args.M) {
            tma_store_2d(&tmC, stage, gcol, row0);          // dgate -> dgu[:, gcol]
            tma_store_2d(&tmC2, stage + 4096, gcol, row0);  // dup -> dgu[:, F + gcol]
            bulk_commit();
          }
          bulk_wait_read0();  // the boxes take the next tile's gate / up values
        }
        __syncwarp();
        if (unit + ustep < total_units) {
          prefetch(unit + ustep);
          inflight = true;
        }
      }
      if (inflight) {  // an aborted run: let the last prefetch land before the CTA exits
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(gb, local & 1)) if (dt_globaltimer() - t0 > 20000000ull) break;
      }
    } else {
    const bool is_bf16 = args.epi == EPI_BF16;
    const int cols_per_box = is_bf16 ? 64 : 32;  // 32 rows x 128 B (bf16) / 32 rows x 128 B (fp32)
    for (int unit = unit0; unit < total_units; unit += ustep, ++local) {
      int tile = unit / args.split_k;
      int mb, nb;
      tile_coords(tile, args.tiles_m, args.tiles_n, mb, nb);
      int acc = local & 1;
      uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&tfull[acc], acc_phase, DT_ERR_TIMEOUT_TMEM, 300, abort_flag)) break;
      tc_fence_after();
      const int row0 = mb * TM + mrow + quad * 32;
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      if constexpr (MODE == 1) {
        // TMEM columns [0, 128): gate, [128, 256): up, for output columns nb*128 + [0, 128); this warp
        // takes output columns [hsel*64, hsel*64 + 64)
        uint8_t* boxA = stage;
        uint8_t* boxB = stage + 4096;
        const int c0 = hsel * 64;
        const int gcol = nb * (BN / 2) + c0;
        const bool live = (gcol < args.N) && (row0 < args.M);
        if (pending) {  // both boxes of the previous tile must have been read out of shared memory
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          pending = false;
        }
        uint32_t hh[2][16];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_row + c0 + 32 * half, g);
          tmem_ld_32x32b_x32(t_row + BN / 2 + c0 + 32 * half, u);
          tmem_ld_wait();
          if (live) {
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
              const uint32_t* gs = g + ch * 8;
              const uint32_t* us = u + ch * 8;
              uint4 vg, vu;
              vg.x = pack_bf16(__uint_as_float(gs[0]), __uint_as_float(gs[1]));
              vg.y = pack_bf16(__uint_as_float(gs[2]), __uint_as_float(gs[3]));
              vg.z = pack_bf16(__uint_as_float(gs[4]), __uint_as_float(gs[5]));
              vg.w = pack_bf16(__uint_as_float(gs[6]), __uint_as_float(gs[7]));
              vu.x = pack_bf16(__uint_as_float(us[0]), __uint_as_float(us[1]));
              vu.y = pack_bf16(__uint_as_float(us[2]), __uint_as_float(us[3]));
              vu.z = pack_bf16(__uint_as_float(us[4]), __uint_as_float(us[5]));
              vu.w = pack_bf16(__uint_as_float(us[6]), __uint_as_float(us[7]));
              box_put(boxA, lane, half * 4 + ch, vg);
              box_put(boxB, lane, half * 4 + ch, vu);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                hh[half][ch * 4 + e] =
                    pack_bf16(silu_f(__uint_as_float(gs[2 * e])) * __uint_as_float(us[2 * e]),
                              silu_f(__uint_as_float(gs[2 * e + 1])) * __uint_as_float(us[2 * e + 1]));
            }
          }
        }
        tc_fence_before();
        arrive_tempty(acc);  // TMEM read; the stores below overlap the next tile's products
        if (live) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, boxA, gcol, row0);   // gate -> gu[:, gcol]
            bulk_commit();
            tma_store_2d(&tmC2, boxB, gcol, row0);  // up -> gu[:, F + gcol]
            bulk_commit();
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");  // box A free again
          }
          __syncwarp();
#pragma unroll
          for (int half = 0; half < 2; ++half)
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
              box_put(boxA, lane, half * 4 + ch,
                      make_uint4(hh[half][ch * 4], hh[half][ch * 4 + 1], hh[half][ch * 4 + 2], hh[half][ch * 4 + 3]));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC3, boxA, gcol, row0);  // h -> h[:, gcol]
            bulk_commit();
          }
          pending = true;
        }
        continue;
      }
      if constexpr (MODE == 3) {
        const int row = row0 + lane;
        const int t = row % args.T;
        const int D = args.hd;
        const float* crow = args.cosT + (long long)t * (D / 2);
        const float* srow = args.sinT + (long long)t * (D / 2);
        // this warp's heads: the half of the tile's columns given by hsel (a whole head when D > BN/2
        // goes to hsel 0)
        const int span = (D <= BN / 2) ? BN / 2 : BN;
        const int h_lo = (D <= BN / 2) ? hsel * span : (hsel ? BN : 0);
#pragma unroll 1
        for (int hc0 = h_lo; hc0 < h_lo + span && hc0 < BN; hc0 += D) {
          const int hc = nb * BN + hc0;  // first output column of this head
          const bool live = (hc < args.N) && (row0 < args.M);
          if (pending) {
            if (lane == 0) bulk_wait_read0();
            __syncwarp();
            pending = false;
          }
          if (!live) continue;
          if (hc < args.rot_cols) {
            // rotate-half pairs (j, j + D/2): 32 pairs per pass
#pragma unroll 1
            for (int j0 = 0; j0 < D / 2; j0 += 32) {
              uint32_t x1[32], x2[32];
              tmem_ld_32x32b_x32(t_row + hc0 + j0, x1);
              tmem_ld_32x32b_x32(t_row + hc0 + D / 2 + j0, x2);
              tmem_ld_wait();
#pragma unroll
              for (int ch = 0; ch < 4; ++ch) {
                const int e0 = j0 + ch * 8;
                const float4 c0 = *reinterpret_cast<const float4*>(crow + e0);
                const float4 c1 = *reinterpret_cast<const float4*>(crow + e0 + 4);
                const float4 s0 = *reinterpret_cast<const float4*>(srow + e0);
                const float4 s1 = *reinterpret_cast<const float4*>(srow + e0 + 4);
                const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                float b1[8], b2[8];
                if (args.bias) {
                  const float4 p0 = *reinterpret_cast<const float4*>(args.bias + hc + e0);
                  const float4 p1 = *reinterpret_cast<const float4*>(args.bias + hc + e0 + 4);
                  const float4 q0 = *reinterpret_cast<const float4*>(args.bias + hc + D / 2 + e0);
                  const float4 q1 = *reinterpret_cast<const float4*>(args.bias + hc + D / 2 + e0 + 4);
                  b1[0] = p0.x; b1[1] = p0.y; b1[2] = p0.z; b1[3] = p0.w;
                  b1[4] = p1.x; b1[5] = p1.y; b1[6] = p1.z; b1[7] = p1.w;
                  b2[0] = q0.x; b2[1] = q0.y; b2[2] = q0.z; b2[3] = q0.w;
                  b2[4] = q1.x; b2[5] = q1.y; b2[6] = q1.z; b2[7] = q1.w;
                } else {
#pragma unroll
                  for (int e = 0; e < 8; ++e) b1[e] = b2[e] = 0.f;
                }
                uint32_t y1[4], y2[4];
#pragma unroll
                for (int e = 0; e < 8; e += 2) {
                  const float a0 = __uint_as_float(x1[ch * 8 + e]) + b1[e];
                  const float a1 = __uint_as_float(x1[ch * 8 + e + 1]) + b1[e + 1];
                  const float q0 = __uint_as_float(x2[ch * 8 + e]) + b2[e];
                  const float q1 = __uint_as_float(x2[ch * 8 + e + 1]) + b2[e + 1];
                  y1[e / 2] = pack_bf16(a0 * cs[e] - q0 * sn[e], a1 * cs[e + 1] - q1 * sn[e + 1]);
                  y2[e / 2] = pack_bf16(a0 * sn[e] + q0 * cs[e], a1 * sn[e + 1] + q1 * cs[e + 1]);
                }
                box_put(stage + (e0 / 64) * 4096, lane, (e0 % 64) / 8, make_uint4(y1[0], y1[1], y1[2], y1[3]));
                box_put(stage + ((D / 2 + e0) / 64) * 4096, lane, ((D / 2 + e0) % 64) / 8,
                        make_uint4(y2[0], y2[1], y2[2], y2[3]));
              }
            }
          } else {
            // v head: bias only
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
              uint32_t x[32];
              tmem_ld_32x32b_x32(t_row + hc0 + c, x);
              tmem_ld_wait();
#pragma unroll
              for (int ch = 0; ch < 4; ++ch) {
                float b[8];
                if (args.bias) {
                  const float4 p0 = *reinterpret_cast<const float4*>(args.bias + hc + c + ch * 8);
                  const float4 p1 = *reinterpret_cast<const float4*>(args.bias + hc + c + ch * 8 + 4);
                  b[0] = p0.x; b[1] = p0.y; b[2] = p0.z; b[3] = p0.w; b[4] = p1.x; b[5] = p1.y; b[6] = p1.z; b[7] = p1.w;
                } else {
#pragma unroll
                  for (int e = 0; e < 8; ++e) b[e] = 0.f;
                }
                uint32_t y[4];
#pragma unroll
                for (int e = 0; e < 8; e += 2)
                  y[e / 2] = pack_bf16(__uint_as_float(x[ch * 8 + e]) + b[e], __uint_as_float(x[ch * 8 + e + 1]) + b[e + 1]);
                box_put(stage + (c / 64) * 4096, lane, (c % 64) / 8 + ch, make_uint4(y[0], y[1], y[2], y[3]));
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stage, hc, row0);
            if (D == 128) tma_store_2d(&tmC, stage + 4096, hc + 64, row0);
            bulk_commit();
          }
          pending = true;
        }
        tc_fence_before();
        arrive_tempty(acc);
        continue;
      }
      if constexpr (MODE == 0 || MODE == 4) {
      // MODE 4: running softmax statistics of this row over this warp's columns (base-2 exponent)
      float st_m = -INFINITY, st_s = 0.f, st_t = 0.f;
      bool st_has_t = false;
      int tgt = -1;
      if constexpr (MODE == 4) {
        const int row = row0 + lane;
        if (row < args.M) {
          const long long grow = args.r0 + row;
          const long long b = grow / args.T, t = grow - b * args.T;
          tgt = args.ids[b * args.S + t + 1];
        }
      }
#pragma unroll 1
      for (int c0 = hsel ? C::COL_SPLIT : 0; c0 < (hsel ? BN : C::COL_SPLIT); c0 += cols_per_box) {
        uint32_t r[2][32];
        tmem_ld_32x32b_x32(t_row + c0, r[0]);
        if (is_bf16) tmem_ld_32x32b_x32(t_row + c0 + 32, r[1]);
        tmem_ld_wait();
        const int gcol = nb * BN + c0;
        const bool live = (gcol < args.N) && (row0 < args.M);
        if constexpr (MODE == 4) {
          const int nv = min(64, args.N - gcol);  // valid columns of this box
          float mx = -INFINITY;
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float v = __uint_as_float(r[e >> 5][e & 31]);
            mx = (e < nv) ? fmaxf(mx, v) : mx;
          }
          if (mx > -INFINITY) {
            const float mn = fmaxf(st_m, mx);
            const float ml2 = mn * 1.4426950408889634f;
            float acc = 0.f;
#pragma unroll
            for (int e = 0; e < 64; ++e) {
              const float v = __uint_as_float(r[e >> 5][e & 31]);
              acc += (e < nv) ? ex2_approx(fmaf(v, 1.4426950408889634f, -ml2)) : 0.f;
            }
            st_s = st_s * ex2_approx((st_m - mn) * 1.4426950408889634f) + acc;
            st_m = mn;
          }
          const int tc = tgt - gcol;
          if (tc >= 0 && tc < 64 && tc < nv) {
            float tv = 0.f;
#pragma unroll
            for (int e = 0; e < 64; ++e) tv = (e == tc) ? __uint_as_float(r[e >> 5][e & 31]) : tv;
            st_t = tv;
            st_has_t = true;
          }
        }
        if (pending) {  // previous box of this warp must have been read out of shared memory
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          pending = false;
        }
        if (live) {
          // row `lane` of the box: 128 bytes as 8 x 16 B chunks in the TMA 128-byte swizzle layout
          // (chunk k stored at k ^ (row & 7)), so the 32 lanes' stores spread over all banks
          uint8_t* rowp = stage + lane * 128;
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            uint4 v;
            if (is_bf16) {
              const uint32_t* src = r[ch >> 2] + (ch & 3) * 8;
              v.x = pack_bf16(__uint_as_float(src[0]) * args.alpha, __uint_as_float(src[1]) * args.alpha);
              v.y = pack_bf16(__uint_as_float(src[2]) * args.alpha, __uint_as_float(src[3]) * args.alpha);
              v.z = pack_bf16(__uint_as_float(src[4]) * args.alpha, __uint_as_float(src[5]) * args.alpha);
              v.w = pack_bf16(__uint_as_float(src[6]) * args.alpha, __uint_as_float(src[7]) * args.alpha);
            } else {
              const uint32_t* src = r[0] + ch * 4;
              v.x = __float_as_uint(__uint_as_float(src[0]) * args.alpha);
              v.y = __float_as_uint(__uint_as_float(src[1]) * args.alpha);
              v.z = __float_as_uint(__uint_as_float(src[2]) * args.alpha);
              v.w = __float_as_uint(__uint_as_float(src[3]) * args.alpha);
            }
            *reinterpret_cast<uint4*>(rowp + ((ch ^ (lane & 7)) * 16)) = v;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (args.epi == EPI_F32_ATOMIC) tma_reduce_add_2d(&tmC, stage, gcol, row0);
            else tma_store_2d(&tmC, stage, gcol, row0);
            if (args.peer) tma_store_2d(&tmCp, stage, gcol, row0);
            bulk_commit();
          }
          pending = true;
        }
      }
      tc_fence_before();
      arrive_tempty(acc);
      if constexpr (MODE == 4) {
        const int row = row0 + lane;
        if (row < args.M) {
          args.lse_part[(long long)(nb * 2 + hsel) * args.M + row] = make_float2(st_m, st_s);
          if (st_has_t) args.tgt_logit[row] = st_t;
        }
      }
      }
    }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // a pair: neither CTA releases TMEM or exits while the other may still signal its barriers or the
  // even CTA's MMAs may still write the odd CTA's TMEM
  if constexpr (PAIR) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_ALLOC);
    else tmem_dealloc(tmem_base, C::TMEM_ALLOC);
  }
  if (args.peer && threadIdx.x == 0) {
    // every epilogue warp has waited for its bulk stores (wait_group 0) before the barrier above
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence_system();
    if (atomicAdd(args.done_ctas, 1u) == gridDim.x - 1) {
      *args.done_ctas = 0u;
      __threadfence_system();
      asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(args.peer_arrivals) : "memory");
    }
  }
}

// ───────────────────────────── host side ─────────────────────────────
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? 0 : -1;
}

// 2-D tensor map over a row-major [outer, inner] matrix with row stride `ld` elements.
int make_map(CUtensorMap* m, const void* ptr, long long inner, long long outer, long long ld, int box_inner,
             int box_outer, bool f32 = false, bool swizzle = true) {
  if (get_encode()) return -2;
  const int esz = f32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

int g_num_sms = 0;

template <int BN, int A_MN, int B_MN, int MODE = 0, bool PAIR = false>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tcp,
           const GemmArgs& a, int grid, cudaStream_t st, const CUtensorMap* tb2 = nullptr,
           const CUtensorMap* tc2 = nullptr, const CUtensorMap* tc3 = nullptr) {
  using C = Cfg<BN, MODE, PAIR>;
  static_assert(C::SMEM_BYTES <= 232448, "shared memory per CTA");
  auto k = gemm_tc_kernel<BN, A_MN, B_MN, MODE, PAIR>;
  static bool attr_set = false;
  if (!attr_set) {
    DT_CUDA_RET(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    attr_set = true;
  }
  if constexpr (PAIR) {
    // clusters of two CTAs (grid even); the pair's SMs share one tile
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    DT_CUDA_RET(cudaLaunchKernelEx(&cfg, k, ta, tb, tc, tcp, tb2 ? *tb2 : tb, tc2 ? *tc2 : tc, tc3 ? *tc3 : tc, a));
    return 0;
  } else {
    k<<<grid, NUM_THREADS, C::SMEM_BYTES, st>>>(ta, tb, tc, tcp, tb2 ? *tb2 : tb, tc2 ? *tc2 : tc, tc3 ? *tc3 : tc, a);
    return (int)cudaGetLastError();
  }
}

// CTA pairs (256-row tiles on two SMs) serve the plain GEMM's 256-wide tiles by default. DT_GEMM_PAIR=0
// turns them off, =1 also routes its 128-wide tiles to pairs (a test setting: slower on every shape of
// the tiny preset). Measured on B200 (256-wide tiles, pairs against single CTAs): LM-head-shaped
// product 0.331 vs 0.358 ms, gate|up-shaped 0.167 vs 0.177, down data-gradient 0.087 vs 0.093, QKV-shaped
// 0.058 vs 0.060, 8192^3 0.765 vs 0.793; N = 768 products unchanged. The fused epilogues (SwiGLU,
// QKV + RoPE, LM head + softmax statistics) stay on single CTAs: paired, a tile waits for the slower of
// two heavy epilogues before its accumulator is reused (SwiGLU forward 0.253 vs 0.222 ms).
int pair_mode() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DT_GEMM_PAIR");
    v = e ? atoi(e) : 2;
  }
  return v;
}
bool use_pair(int bn) { return bn == 256 ? pair_mode() >= 1 : (bn == 128 && pair_mode() == 1); }

int num_sms() {
  if (!g_num_sms) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return g_num_sms;
}
int pair_grid(int units) {
  const int pairs = units < num_sms() / 2 ? units : num_sms() / 2;
  return 2 * pairs;
}

}  // namespace

namespace {
int gemm_impl(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, void* Cp, long long ldc,
              int M, int N, int K, int epi, float alpha, int split_k, int bn, void* Cpeer, unsigned* peer_arrivals,
              unsigned* done_ctas, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((lda % 8) || (ldb % 8) || ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15)) return -10;
  if (split_k > 1 && epi != EPI_F32_ATOMIC) return -11;
  if (!g_num_sms) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  }
  if (bn != 128 && bn != 192 && bn != 256) {
    // pick the N tile by wave quantisation: rounds of the persistent grid x the relative cost of one tile
    // (128 wide ~0.65, 192 wide ~0.82 of a 256-wide one: the A tile and the per-tile fixed work stay)
    long long tm = (M + BM - 1) / BM;
    auto rounds = [&](int w) { return (tm * ((N + w - 1) / w) + g_num_sms - 1) / g_num_sms; };
    const long long c256 = rounds(256) * 100, c128 = rounds(128) * 65;
    const long long c192 = (N >= 384 && N % 192 == 0 && !Cpeer) ? rounds(192) * 82 : (1LL << 60);
    bn = N <= 128 ? 128 : (c128 < c256 && c128 < c192 ? 128 : (c192 < c256 ? 192 : 256));
    // accumulate / split-K problems fill the machine through K splits instead: keep the wide tile
    if (epi == EPI_F32_ATOMIC && N > 128 && tm * ((N + 255) / 256) < g_num_sms) bn = 256;
  }
  const bool pair = use_pair(bn);
  GemmArgs a = {};
  a.M = M; a.N = N; a.K = K;
  a.num_kb = (K + BK - 1) / BK;
  a.tiles_m = (M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM);
  a.tiles_n = (N + bn - 1) / bn;
  int tiles = a.tiles_m * a.tiles_n;
  if (split_k <= 0) {
    // Auto split-K (accumulating epilogue only): the smallest split whose work units fill >= 90 % of the
    // last wave of the persistent grid (units / (waves * SMs)), keeping >= 8 K-blocks per split; without
    // one, the split with the best fill. A power-of-two rule lands e.g. 96 tiles on 192 units = 1.3 waves.
    split_k = 1;
    if (epi == EPI_F32_ATOMIC) {
      const int slots = pair ? g_num_sms / 2 : g_num_sms;
      auto fill = [&](int sk) {
        const long long u = (long long)tiles * sk;
        return (double)u / (double)(((u + slots - 1) / slots) * slots);
      };
      int best = 1;
      double best_fill = fill(1);
      for (int sk = 1; sk <= 32 && a.num_kb / sk >= 8; ++sk) {
        const double f = fill(sk);
        if (f >= 0.9) { best = sk; break; }
        if (f > best_fill + 1e-9) { best = sk; best_fill = f; }
      }
      split_k = best;
    }
  }
  split_k = split_k < 1 ? 1 : (split_k > a.num_kb ? a.num_kb : split_k);
  a.kb_per_split = (a.num_kb + split_k - 1) / split_k;
  a.split_k = (a.num_kb + a.kb_per_split - 1) / a.kb_per_split;
  a.epi = epi;
  a.alpha = alpha;
  a.C = Cp;
  a.ldc = ldc;
  a.peer = Cpeer != nullptr;
  a.peer_arrivals = peer_arrivals;
  a.done_ctas = done_ctas;
  if (a.peer && (epi != EPI_BF16 || !peer_arrivals || !done_ctas || (reinterpret_cast<uintptr_t>(Cpeer) & 15)))
    return -13;

  if ((ldc % (epi == EPI_BF16 ? 8 : 4)) || (reinterpret_cast<uintptr_t>(Cp) & 15)) return -12;
  CUtensorMap ta, tb, tcm, tcp;
  int rc;
  rc = (epi == EPI_BF16) ? make_map(&tcm, Cp, N, M, ldc, 64, 32, false, true)
                         : make_map(&tcm, Cp, N, M, ldc, 32, 32, true, true);
  if (rc) return rc;
  tcp = tcm;
  if (a.peer && (rc = make_map(&tcp, Cpeer, N, M, ldc, 64, 32, false, true))) return rc;
  rc = a_mn ? make_map(&ta, A, M, K, lda, 64, BK) : make_map(&ta, A, K, M, lda, BK, BM);
  if (rc) return rc;
  rc = b_mn ? make_map(&tb, B, N, K, ldb, 64, BK) : make_map(&tb, B, K, N, ldb, BK, pair ? bn / 2 : bn);
  if (rc) return rc;

  int units = tiles * a.split_k;
  if (pair) {
    const int grid2 = pair_grid(units);
    if (bn == 256) {
      if (!a_mn && !b_mn) return launch<256, 0, 0, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
      if (!a_mn && b_mn) return launch<256, 0, 1, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
      if (a_mn && !b_mn) return launch<256, 1, 0, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
      return launch<256, 1, 1, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
    }
    if (!a_mn && !b_mn) return launch<128, 0, 0, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
    if (!a_mn && b_mn) return launch<128, 0, 1, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
    if (a_mn && !b_mn) return launch<128, 1, 0, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
    return launch<128, 1, 1, 0, true>(ta, tb, tcm, tcp, a, grid2, stream);
  }
  int grid = units < g_num_sms ? units : g_num_sms;
  if (bn == 256) {
    if (!a_mn && !b_mn) return launch<256, 0, 0>(ta, tb, tcm, tcp, a, grid, stream);
    if (!a_mn && b_mn) return launch<256, 0, 1>(ta, tb, tcm, tcp, a, grid, stream);
    if (a_mn && !b_mn) return launch<256, 1, 0>(ta, tb, tcm, tcp, a, grid, stream);
    return launch<256, 1, 1>(ta, tb, tcm, tcp, a, grid, stream);
  } else if (bn == 192) {
    if (!a_mn && !b_mn) return launch<192, 0, 0>(ta, tb, tcm, tcp, a, grid, stream);
    if (!a_mn && b_mn) return launch<192, 0, 1>(ta, tb, tcm, tcp, a, grid, stream);
    if (a_mn && !b_mn) return launch<192, 1, 0>(ta, tb, tcm, tcp, a, grid, stream);
    return launch<192, 1, 1>(ta, tb, tcm, tcp, a, grid, stream);
  } else {
    if (!a_mn && !b_mn) return launch<128, 0, 0>(ta, tb, tcm, tcp, a, grid, stream);
    if (!a_mn && b_mn) return launch<128, 0, 1>(ta, tb, tcm, tcp, a, grid, stream);
    if (a_mn && !b_mn) return launch<128, 1, 0>(ta, tb, tcm, tcp, a, grid, stream);
    return launch<128, 1, 1>(ta, tb, tcm, tcp, a, grid, stream);
  }
}
}  // namespace

// C[M,N] (op)= alpha * A[M,K] . B[N,K]^T
//   a_mn = 0: A(m,k) at A[m*lda + k];  a_mn = 1: A(m,k) at A[k*lda + m]
//   b_mn = 0: B(n,k) at B[n*ldb + k];  b_mn = 1: B(n,k) at B[k*ldb + n]
//   epi: 0 bf16 store, 1 fp32 store, 2 fp32 atomic add;  split_k > 1 requires epi == 2.
//   bn: 128, 192 or 256 (0 = choose).  Returns 0 or a CUDA / argument error code.
DT_API int dt_gemm_bf16(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, void* Cp,
                        long long ldc, int M, int N, int K, int epi, float alpha, int split_k, int bn,
                        cudaStream_t stream) {
  return gemm_impl(A, a_mn, lda, B, b_mn, ldb, Cp, ldc, M, N, K, epi, alpha, split_k, bn, nullptr, nullptr, nullptr,
                   stream);
}

// Same product (bf16 epilogue) whose every output box is also stored into `Cpeer` (a peer GPU's buffer of
// the same shape and ldc, mapped into this process); when all boxes have landed the kernel adds 1 to
// *peer_arrivals (on the peer) with a system-scope release. `done_ctas` is a zeroed local counter.
DT_API int dt_gemm_bf16_peer(const void* A, int a_mn, long long lda, const void* B, int b_mn, long long ldb, void* Cp,
                             long long ldc, int M, int N, int K, float alpha, int bn, void* Cpeer,
                             unsigned* peer_arrivals, unsigned* done_ctas, cudaStream_t stream) {
  return gemm_impl(A, a_mn, lda, B, b_mn, ldb, Cp, ldc, M, N, K, EPI_BF16, alpha, 1, bn, Cpeer, peer_arrivals,
                   done_ctas, stream);
}

// ───────────────────────────── fused SwiGLU ─────────────────────────────
// Forward: X [M, K] (row stride ldx) times the gate|up weight Wgu [2F, K] (row stride ldw; gate rows
// [0, F), up rows [F, 2F)). Writes gu [M, 2F] (gate | up, bf16, for the backward) and h = silu(gate) * up
// [M, F] (bf16, computed from the fp32 accumulators). F must be a multiple of 64.
DT_API int dt_gemm_swiglu_fwd(const void* X, long long ldx, const void* Wgu, long long ldw, void* gu, void* h,
                              int M, int F, int K, cudaStream_t stream) {
  if (M <= 0 || F <= 0 || K <= 0) return 0;
  if ((F % 64) || (ldx % 8) || (ldw % 8) ||
      ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(Wgu) | reinterpret_cast<uintptr_t>(gu) |
        reinterpret_cast<uintptr_t>(h)) & 15))
    return -10;
  GemmArgs a = {};
  a.M = M; a.N = F; a.K = K;
  a.num_kb = (K + BK - 1) / BK;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (F + 127) / 128;
  a.split_k = 1;
  a.kb_per_split = a.num_kb;
  a.epi = EPI_BF16;
  a.alpha = 1.f;
  a.C = gu;
  a.ldc = 2LL * F;
  const __nv_bfloat16* wup = reinterpret_cast<const __nv_bfloat16*>(Wgu) + (long long)F * ldw;
  __nv_bfloat16* gu_up = reinterpret_cast<__nv_bfloat16*>(gu) + F;
  CUtensorMap ta, tb, tb2, tc, tc2, tc3;
  int rc;
  if ((rc = make_map(&ta, X, K, M, ldx, BK, BM))) return rc;
  if ((rc = make_map(&tb, Wgu, K, F, ldw, BK, 128))) return rc;
  if ((rc = make_map(&tb2, wup, K, F, ldw, BK, 128))) return rc;
  if ((rc = make_map(&tc, gu, F, M, 2LL * F, 64, 32))) return rc;
  if ((rc = make_map(&tc2, gu_up, F, M, 2LL * F, 64, 32))) return rc;
  if ((rc = make_map(&tc3, h, F, M, F, 64, 32))) return rc;
  const int tiles = a.tiles_m * a.tiles_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return launch<256, 0, 0, 1>(ta, tb, tc, tc, a, grid, stream, &tb2, &tc2, &tc3);
}

// Backward through SwiGLU and the down projection's input: dh = dY [M, K] . Wd [K, F] (row stride ldw),
// never stored; with the saved gu [M, 2F] of the forward, writes dgu[:, :F] = dh * up * silu'(gate) and
// dgu[:, F:] = dh * silu(gate) (bf16). F must be a multiple of 64; 128-wide tiles (`bn` is ignored).
DT_API int dt_gemm_swiglu_bwd(const void* dY, long long ldy, const void* Wd, long long ldw, const void* gu, void* dgu,
                              int M, int F, int K, int bn, cudaStream_t stream) {
  (void)bn;
  if (M <= 0 || F <= 0 || K <= 0) return 0;
  if ((F % 64) || (ldy % 8) || (ldw % 8) ||
      ((reinterpret_cast<uintptr_t>(dY) | reinterpret_cast<uintptr_t>(Wd) | reinterpret_cast<uintptr_t>(gu) |
        reinterpret_cast<uintptr_t>(dgu)) & 15))
    return -10;
  constexpr int kBN = 128;
  GemmArgs a = {};
  a.M = M; a.N = F; a.K = K;
  a.num_kb = (K + BK - 1) / BK;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (F + kBN - 1) / kBN;
  a.split_k = 1;
  a.kb_per_split = a.num_kb;
  a.epi = EPI_BF16;
  a.alpha = 1.f;
  a.C = dgu;
  a.ldc = 2LL * F;
  const __nv_bfloat16* gu_up = reinterpret_cast<const __nv_bfloat16*>(gu) + F;
  __nv_bfloat16* dgu_up = reinterpret_cast<__nv_bfloat16*>(dgu) + F;
  CUtensorMap ta, tb, tc, tc2, tg, tu;
  int rc;
  if ((rc = make_map(&ta, dY, K, M, ldy, BK, BM))) return rc;
  if ((rc = make_map(&tb, Wd, F, K, ldw, 64, BK))) return rc;  // B(n, k) = Wd[k * ldw + n]: MN-major
  if ((rc = make_map(&tc, dgu, F, M, 2LL * F, 64, 32))) return rc;
  if ((rc = make_map(&tc2, dgu_up, F, M, 2LL * F, 64, 32))) return rc;
  if ((rc = make_map(&tg, gu, F, M, 2LL * F, 64, 32))) return rc;      // saved gate, read by the epilogue
  if ((rc = make_map(&tu, gu_up, F, M, 2LL * F, 64, 32))) return rc;   // saved up
  const int tiles = a.tiles_m * a.tiles_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return launch<kBN, 0, 1, 2>(ta, tb, tc, tc, a, grid, stream, &tg, &tc2, &tu);
}

// ───────────────────────────── fused QKV bias + RoPE ─────────────────────────────
// out[M, N] = X [M, K] . Wqkv [N, K]^T + bias, then the rotate-half rotary embedding of every head whose
// first column is below rot_cols (the q and k heads), position = row mod T, tables cos / sin [T, hd/2]
// fp32; hd 64 or 128 and N a multiple of hd. bias may be null. bn 128 / 256 (0 = choose).
DT_API int dt_gemm_qkv_rope(const void* X, long long ldx, const void* Wqkv, long long ldw, const float* bias,
                            const float* cosT, const float* sinT, void* out, int M, int N, int K, int T, int hd,
                            int rot_cols, int bn, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((hd != 64 && hd != 128) || (N % hd) || (rot_cols % hd) || T <= 0 || (ldx % 8) || (ldw % 8) ||
      ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(Wqkv) | reinterpret_cast<uintptr_t>(out) |
        reinterpret_cast<uintptr_t>(cosT) | reinterpret_cast<uintptr_t>(sinT) | reinterpret_cast<uintptr_t>(bias)) & 15))
    return -10;
  if (bn != 128 && bn != 256) {
    const long long tm = (M + BM - 1) / BM;
    const long long w256 = (tm * ((N + 255) / 256) + num_sms() - 1) / num_sms();
    const long long w128 = (tm * ((N + 127) / 128) + num_sms() - 1) / num_sms();
    bn = (N <= 128 || w128 * 65 < w256 * 100) ? 128 : 256;
  }
  if (hd == 128) bn = 256;  // one 128-wide head per epilogue warp pair half
  GemmArgs a = {};
  a.M = M; a.N = N; a.K = K;
  a.num_kb = (K + BK - 1) / BK;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (N + bn - 1) / bn;
  a.split_k = 1;
  a.kb_per_split = a.num_kb;
  a.epi = EPI_BF16;
  a.alpha = 1.f;
  a.C = out;
  a.ldc = N;
  a.cosT = cosT;
  a.sinT = sinT;
  a.bias = bias;
  a.T = T;
  a.hd = hd;
  a.rot_cols = rot_cols;
  CUtensorMap ta, tb, tc;
  int rc;
  if ((rc = make_map(&ta, X, K, M, ldx, BK, BM))) return rc;
  if ((rc = make_map(&tb, Wqkv, K, N, ldw, BK, bn))) return rc;
  if ((rc = make_map(&tc, out, N, M, N, 64, 32))) return rc;
  const int tiles = a.tiles_m * a.tiles_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  if (bn == 256) return launch<256, 0, 0, 3>(ta, tb, tc, tc, a, grid, stream);
  return launch<128, 0, 0, 3>(ta, tb, tc, tc, a, grid, stream);
}

// ───────────────────────────── LM head with softmax statistics ─────────────────────────────
// logits[rows, V] (bf16, row stride ldc) = X [rows, K] . E [V, K]^T, plus lse_part[(2 * tile_n + half) *
// rows + row] = (max, sum exp(x - max)) of the fp32 logits over each half of each 256-wide column tile and
// tgt_logit[row] = the fp32 logit of ids[b*S + t + 1] for global row r0 + row (b, t = divmod(r0 + row, T)).
// lse_part needs 2 * ceil(V / 256) * rows entries. Returns that count through *n_part when non-null.
DT_API int dt_gemm_logits_lse(const void* X, long long ldx, const void* E, long long lde, void* logits, long long ldc,
                              int rows, int V, int K, float2* lse_part, float* tgt_logit, const int* ids, int T, int S,
                              long long r0, cudaStream_t stream) {
  if (rows <= 0 || V <= 0 || K <= 0) return 0;
  if ((ldx % 8) || (lde % 8) || (ldc % 8) || !lse_part || !tgt_logit || !ids || T <= 0 || S <= T ||
      ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(E) | reinterpret_cast<uintptr_t>(logits)) & 15))
    return -10;
  constexpr int kBN = 256;
  GemmArgs a = {};
  a.M = rows; a.N = V; a.K = K;
  a.num_kb = (K + BK - 1) / BK;
  a.tiles_m = (rows + BM - 1) / BM;
  a.tiles_n = (V + kBN - 1) / kBN;
  a.split_k = 1;
  a.kb_per_split = a.num_kb;
  a.epi = EPI_BF16;
  a.alpha = 1.f;
  a.C = logits;
  a.ldc = ldc;
  a.lse_part = lse_part;
  a.tgt_logit = tgt_logit;
  a.ids = ids;
  a.T = T;
  a.S = S;
  a.r0 = r0;
  CUtensorMap ta, tb, tc;
  int rc;
  if ((rc = make_map(&ta, X, K, rows, ldx, BK, BM))) return rc;
  if ((rc = make_map(&tb, E, K, V, lde, BK, kBN))) return rc;
  if ((rc = make_map(&tc, logits, V, rows, ldc, 64, 32))) return rc;
  const int tiles = a.tiles_m * a.tiles_n;
  const int grid = tiles < num_sms() ? tiles : num_sms();
  return launch<kBN, 0, 0, 4>(ta, tb, tc, tc, a, grid, stream);
}

DT_API long long dt_logits_lse_parts(int rows, int V) { return 2LL * ((V + 255) / 256) * rows; }
