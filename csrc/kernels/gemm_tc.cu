// Persistent tcgen05 GEMM for sm_100a:   C[M,N] (op)= alpha * sum_k A[m,k] * B[n,k]
//
// * Operands are bf16 in global memory, staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, no
//   cluster multicast) into a STAGES-deep shared-memory ring; each operand may be K-major
//   (k contiguous) or MN-major (m / n contiguous), which covers forward (X W^T), data-gradient
//   (dY W) and weight-gradient (dY^T X) products without any transpose pass.
// * One elected thread of warp 1 issues tcgen05.mma (M=128, N=BN, K=16, fp32 accumulate) into one
//   of two TMEM accumulators; tcgen05.commit releases shared-memory stages and hands finished
//   accumulators to the epilogue, so the epilogue of tile i overlaps the main loop of tile i+1.
// * Warps 2..5 drain TMEM with tcgen05.ld (32 lanes x 32 columns per load) into a swizzled shared
//   staging box and write it with a TMA store (bf16 / fp32) or a TMA reduce-add (fp32 accumulation,
//   used for split-K and gradient accumulation), so global writes are full-line and asynchronous.
// * Tiles are visited by a persistent grid (one CTA per SM) in grouped order for L2 reuse.
// Every mbarrier wait is bounded (common.cuh); on timeout the CTA drains its in-flight TMA loads and
// MMAs, frees TMEM and returns with dt_error_word set.
#include "common.cuh"
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int NUM_THREADS = 192;
constexpr int GROUP_M = 16;

enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_F32_ATOMIC = 2 };

struct GemmArgs {
  int M, N, K;
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

template <int BN>
struct Cfg {
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int EPI_BYTES = 4 * 4096;  // one 4 KB staging box per epilogue warp
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;
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

template <int BN, int A_MN, int B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmCp, GemmArgs args) {
  using C = Cfg<BN>;
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *consumed = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_units = args.tiles_m * args.tiles_n * args.split_k;

  if (warp == 0) {
    // ───────────── TMA producer ─────────────
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      int issued = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < total_units && ok; unit += gridDim.x) {
        int s = unit % args.split_k, tile = unit / args.split_k;
        int mb, nb;
        tile_coords(tile, args.tiles_m, args.tiles_n, mb, nb);
        int m0 = mb * BM, n0 = nb * BN;
        int kb0 = s * args.kb_per_split, kb1 = min(kb0 + args.kb_per_split, args.num_kb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, DT_ERR_TIMEOUT_EMPTY, 100, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          if (A_MN) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * (64 * BK * 2), &tmA, &full[stage], m0 + 64 * j, kb * BK);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * BK, m0);
          }
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * (64 * BK * 2), &tmB, &full[stage], n0 + 64 * j, kb * BK);
          } else {
            tma_load_2d(b_dst, &tmB, &full[stage], kb * BK, n0);
          }
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag) {
        // Drain: wait (bounded) for every issued-but-unconsumed stage so no TMA write lands after exit.
        for (int i = *consumed; i < issued; ++i) {
          uint64_t t0 = dt_globaltimer();
          while (!mbar_try_wait(&full[i % C::STAGES], (i / C::STAGES) & 1)) {
            if (dt_globaltimer() - t0 > 20000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ───────────── MMA issuer ─────────────
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      for (int unit = blockIdx.x; unit < total_units && ok; unit += gridDim.x, ++local) {
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
            umma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (!ok && issued_any) {
        // Make sure every issued MMA has retired before TMEM is released.
        umma_commit(drain);
        uint64_t t0 = dt_globaltimer();
        while (!mbar_try_wait(drain, 0)) {
          if (dt_globaltimer() - t0 > 20000000ull) break;
        }
      }
    }
  } else {
    // ───────────── Epilogue: warps 2..5 ─────────────
    // TMEM -> registers (tcgen05.ld, this warp's 32 lanes = 32 tile rows) -> 4 KB shared staging box ->
    // TMA store (bf16 / fp32) or TMA reduce-add (fp32 accumulate); the tensor map clips the M/N tails.
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    uint8_t* stage = sEpi + quad * 4096;
    const bool is_bf16 = args.epi == EPI_BF16;
    const int cols_per_box = is_bf16 ? 64 : 32;  // 32 rows x 128 B (bf16) / 32 rows x 128 B (fp32)
    int local = 0;
    bool pending = false;
    for (int unit = blockIdx.x; unit < total_units; unit += gridDim.x, ++local) {
      int tile = unit / args.split_k;
      int mb, nb;
      tile_coords(tile, args.tiles_m, args.tiles_n, mb, nb);
      int acc = local & 1;
      uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&tfull[acc], acc_phase, DT_ERR_TIMEOUT_TMEM, 300, abort_flag)) break;
      tc_fence_after();
      const int row0 = mb * BM + quad * 32;
      const uint32_t t_row = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += cols_per_box) {
        uint32_t r[2][32];
        tmem_ld_32x32b_x32(t_row + c0, r[0]);
        if (is_bf16) tmem_ld_32x32b_x32(t_row + c0 + 32, r[1]);
        tmem_ld_wait();
        const int gcol = nb * BN + c0;
        const bool live = (gcol < args.N) && (row0 < args.M);
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
      mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
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

template <int BN, int A_MN, int B_MN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tcp,
           const GemmArgs& a, int grid, cudaStream_t st) {
  using C = Cfg<BN>;
  auto k = gemm_tc_kernel<BN, A_MN, B_MN>;
  static bool attr_set = false;
  if (!attr_set) {
    DT_CUDA_RET(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    attr_set = true;
  }
  k<<<grid, NUM_THREADS, C::SMEM_BYTES, st>>>(ta, tb, tc, tcp, a);
  return (int)cudaGetLastError();
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
  if (bn != 128 && bn != 256) {
    // pick the N tile by wave quantisation; a 128-wide tile costs ~0.65 of a 256-wide one (the A tile
    // and the per-tile epilogue are the same size), measured on the tiny-preset shapes
    long long tm = (M + BM - 1) / BM;
    long long w256 = (tm * ((N + 255) / 256) + g_num_sms - 1) / g_num_sms;
    long long w128 = (tm * ((N + 127) / 128) + g_num_sms - 1) / g_num_sms;
    bn = (N <= 128 || w128 * 65 < w256 * 100) ? 128 : 256;
    // accumulate / split-K problems fill the machine through K splits instead: keep the wide tile
    if (epi == EPI_F32_ATOMIC && N > 128 && tm * ((N + 255) / 256) < g_num_sms) bn = 256;
  }
  GemmArgs a;
  a.M = M; a.N = N; a.K = K;
  a.num_kb = (K + BK - 1) / BK;
  a.tiles_m = (M + BM - 1) / BM;
  a.tiles_n = (N + bn - 1) / bn;
  int tiles = a.tiles_m * a.tiles_n;
  if (split_k <= 0) {
    // Auto split-K (accumulating epilogue only): the smallest split whose work units fill >= 90 % of the
    // last wave of the persistent grid (units / (waves * SMs)), keeping >= 8 K-blocks per split; without
    // one, the split with the best fill. A power-of-two rule lands e.g. 96 tiles on 192 units = 1.3 waves.
    split_k = 1;
    if (epi == EPI_F32_ATOMIC) {
      auto fill = [&](int sk) {
        const long long u = (long long)tiles * sk;
        return (double)u / (double)(((u + g_num_sms - 1) / g_num_sms) * g_num_sms);
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
  rc = b_mn ? make_map(&tb, B, N, K, ldb, 64, BK) : make_map(&tb, B, K, N, ldb, BK, bn);
  if (rc) return rc;

  int units = tiles * a.split_k;
  int grid = units < g_num_sms ? units : g_num_sms;
  if (bn == 256) {
    if (!a_mn && !b_mn) return launch<256, 0, 0>(ta, tb, tcm, tcp, a, grid, stream);
    if (!a_mn && b_mn) return launch<256, 0, 1>(ta, tb, tcm, tcp, a, grid, stream);
    if (a_mn && !b_mn) return launch<256, 1, 0>(ta, tb, tcm, tcp, a, grid, stream);
    return launch<256, 1, 1>(ta, tb, tcm, tcp, a, grid, stream);
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
//   bn: 128 or 256 (0 = choose).  Returns 0 or a CUDA / argument error code.
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
