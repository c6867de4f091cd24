// Coordinator merge over device memory (reference coordinator/src/aggregation.rs:255-380):
//
//   pre-pass   per contribution: ||decoded delta||^2, max|x|, non-finite count   (validate_delta,
//              compression.rs:388-424, and the 3x running-average norm clip inputs, aggregation.rs:310-328)
//   accumulate dst[idx] += coef_c * q * scale[blk]   for every kept entry of every accepted contribution,
//              coef_c = clip_c * w_c / sum(w) with w_c = tokens_c * 0.9^staleness_c (weighted_average_gpu,
//              aggregation.rs:28-61). Payloads are read with plain loads straight out of each node's
//              GPU memory (peer pointers of a symmetric allocation, NVLink P2P) - no staging copy.
//              Without outer momentum (the reference's setting, aggregation.rs:364) dst is the checkpoint
//              itself and coef_c carries the factor -outer_lr: theta -= lr * merged delta, in place, with
//              no dense accumulator.
//   broadcast  the new fp32 checkpoint into every node's staging buffer: one multimem.st per 16 bytes
//              through an NVLS multicast object (or one store per peer when no multicast object exists).
//   apply      (outer momentum only) v' = mu*v + acc ; theta -= lr*(mu*v' + acc) (nesterov_step_gpu,
//              aggregation.rs:64-105) fused with the broadcast; acc is cleared.
#include "common.cuh"
#include <cstring>

namespace {

struct Contrib {
  const int* idx;            // kept indices, relative to their 2^31-element window (sparse), or null (dense)
  const signed char* q;      // int8 values (quantised) or null
  const float* val;          // fp32 values (unquantised sparse, or dense delta)
  const float* scales;       // per-block scales (quantised)
  const long long* win;      // position where each index window starts (8 entries) or null (one window)
  long long count;           // kept entries (sparse) or length (dense)
  int block;                 // quantisation block
  int dense;
  float coef;                // weight / total * clip scale
  int pad;
};
static_assert(sizeof(Contrib) == 64, "Contrib layout is shared with the host packer");

// The descriptor table travels as a kernel parameter (64 x 64 B; kernel parameters up to 32 KB): it is
// captured at launch, so no device copy of it can be read before its upload has landed.
constexpr int MAX_CONTRIB = 64;
struct ContribTable {
  Contrib c[MAX_CONTRIB];
};

constexpr int MUNR = 4;

// Window starts of a contribution (positions; int64 max = none), loaded once per thread.
struct Windows {
  long long start[7];  // starts of windows 1..7
  int n;               // how many of them exist
  __device__ __forceinline__ void load(const long long* win) {
    n = 0;
    if (!win) return;
#pragma unroll
    for (int k = 0; k < 7; ++k) {
      start[k] = __ldg(win + 1 + k);
      if (start[k] != 0x7fffffffffffffffLL) n = k + 1;
    }
  }
  // flat index of the entry at position p
  __device__ __forceinline__ long long flat(int idx, long long p) const {
    long long w = 0;
    for (int k = 0; k < n; ++k) w += p >= start[k];
    return (long long)idx + (w << 31);
  }
};

__device__ __forceinline__ float contrib_value(const Contrib& c, long long i) {
  if (c.q) {
    // power-of-two blocks (the usual 256) by shift: a 64-bit division costs dozens of instructions per entry
    const long long blk = (c.block & (c.block - 1)) == 0 ? (i >> (__ffs(c.block) - 1)) : i / c.block;  // block >= 1
    return (float)__ldg(c.q + i) * __ldg(c.scales + blk);
  }
  return __ldg(c.val + i);
}

__global__ void prepass_kernel(const __grid_constant__ ContribTable cs, int n, double* __restrict__ stats) {
  // grid: (blocks per contribution, n); stats[c*3 + {sumsq, maxabs, nonfinite}]
  __shared__ float shs[32];
  const int c = blockIdx.y;
  const Contrib& C = cs.c[c];
  float ss = 0.f, mx = 0.f;
  int nf = 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  // MUNR independent elements per thread per iteration: all loads in flight before any use
  for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < C.count; i0 += stride * MUNR) {
    float v[MUNR];
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      v[u] = i < C.count ? contrib_value(C, i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      if (!isfinite(v[u])) { nf = 1; continue; }
      ss += v[u] * v[u];
      mx = fmaxf(mx, fabsf(v[u]));
    }
  }
  float t = block_sum(ss, shs);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned long long*>(stats + c * 3 + 1),
                                         (unsigned long long)__double_as_longlong((double)mx));
  nf = __syncthreads_or(nf);
  if (threadIdx.x == 0) {
    atomicAdd(stats + c * 3 + 0, (double)t);
    if (nf) atomicAdd(stats + c * 3 + 2, 1.0);
  }
}

__global__ void accumulate_kernel(const __grid_constant__ ContribTable cs, int n, float* __restrict__ acc) {
  const int c = blockIdx.y;
  const Contrib& C = cs.c[c];
  if (C.coef == 0.f) return;
  if (C.dense) {
    const long long n4 = C.count / 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
      float4 v = __ldg(reinterpret_cast<const float4*>(C.val) + i);
      atomicAdd(reinterpret_cast<float4*>(acc) + i, make_float4(v.x * C.coef, v.y * C.coef, v.z * C.coef, v.w * C.coef));
    }
    for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < C.count;
         i += (long long)gridDim.x * blockDim.x)
      atomicAdd(acc + i, __ldg(C.val + i) * C.coef);
    return;
  }
  Windows W;
  W.load(C.win);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < C.count; i0 += stride * MUNR) {
    int j[MUNR];
    float v[MUNR];
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      j[u] = i < C.count ? __ldg(C.idx + i) : -1;
      v[u] = i < C.count ? contrib_value(C, i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < MUNR; ++u)
      if (j[u] >= 0) atomicAdd(acc + W.flat(j[u], i0 + u * stride), v[u] * C.coef);
  }
}

__device__ __forceinline__ void mc_store_v4(void* mc_addr, float4 v) {
  asm volatile("multimem.st.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

struct Dests {
  float* stage32[8];
  int n;
};

__device__ __forceinline__ void store_dests(float* mc32, const Dests& d, const float* self, long long i, float4 t) {
  if (mc32) {
    mc_store_v4(reinterpret_cast<float4*>(mc32) + i, t);
  } else {
    for (int r = 0; r < d.n; ++r)
      if (d.stage32[r] != self) reinterpret_cast<float4*>(d.stage32[r])[i] = t;
  }
}

// theta, vel, acc: local fp32 [n] (n a multiple of 4). Broadcast targets: a multicast address (mc32
// non-null) or per-peer pointers in `d`.
__global__ void apply_broadcast_kernel(float* __restrict__ theta, float* __restrict__ vel, float* __restrict__ acc,
                                       long long n, float lr, float mu, float* mc32, Dests d) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 a = reinterpret_cast<float4*>(acc)[i];
    float4 t = reinterpret_cast<float4*>(theta)[i];
    float* ap = &a.x;
    float* tp = &t.x;
    if (vel) {
      float4 v = reinterpret_cast<float4*>(vel)[i];
      float* vp = &v.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        vp[k] = mu * vp[k] + ap[k];
        tp[k] -= lr * (mu * vp[k] + ap[k]);
      }
      reinterpret_cast<float4*>(vel)[i] = v;
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) tp[k] -= lr * ap[k];
    }
    reinterpret_cast<float4*>(theta)[i] = t;
    reinterpret_cast<float4*>(acc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    store_dests(mc32, d, theta, i, t);
  }
  __threadfence_system();
}

// theta (already updated in place) -> every node's staging buffer. When theta is this GPU's own staging
// buffer, the multicast store rewrites the local copy with the value just read from it.
__global__ void broadcast_kernel(const float* __restrict__ theta, long long n, float* mc32, Dests d) {
  const long long n4 = n / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < n4; i0 += stride * MUNR) {
    float4 t[MUNR];
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      if (i < n4) t[u] = reinterpret_cast<const float4*>(theta)[i];
    }
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      if (i < n4) store_dests(mc32, d, theta, i, t[u]);
    }
  }
  __threadfence_system();
}

// ───────────── distributed merge: every node merges one slice of the flat range ─────────────
// Node r owns the flat range [a_r, b_r) (float4-aligned, about n/W elements). Rank 0 plans the attempt on
// the host from the statistics every node reported with its push (validation, clipping, weights) and
// announces members and coefficients; then every node:
//   dm_range    finds, per sparse member payload, the positions whose flat index falls in its range
//               (payload indices ascend, so a 32-ary warp search over the peer's index array);
//   dm_apply    adds coef * x into its slice of the checkpoint (its own staging slot) - dense members
//               fused in one pass, sparse ones by atomics;
//   dm_broadcast writes its slice into every node's slot (multimem.st, or one store per peer) and
//               releases rank 0's done counter.
// Each payload is read once, by the node that owns the slice. Cross-node ordering is on the host (the
// announcement before the kernels, a completion key after them); rank 0's final bounded wait on the
// done counter (target att * W, counters only grow) checks that every slice landed.
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Bounded wait by one thread until *p >= target; false on timeout (error recorded at `site`).
__device__ __forceinline__ bool wait_ge_u64(const unsigned long long* p, unsigned long long target, int site,
                                           unsigned long long bound_ns = DT_WAIT_NS) {
  if (ld_acquire_sys_u64(p) >= target) return true;
  const uint64_t t0 = dt_globaltimer();
  while (ld_acquire_sys_u64(p) < target) {
    if (*reinterpret_cast<volatile int*>(&dt_error_word) != 0 || dt_globaltimer() - t0 > bound_ns) {
      dt_set_error(DT_ERR_TIMEOUT_PEER, site);
      return false;
    }
  }
  return true;
}

// First position p in [0, count) with flat(p) >= x (count if none), by one warp.
__device__ long long warp_lower_bound(const Contrib& C, const Windows& W, long long x) {
  const int lane = threadIdx.x & 31;
  long long L = 0, R = C.count;
  while (R - L > 32) {
    const long long step = (R - L + 31) / 32;
    const long long p = L + lane * step;
    const bool ge = p >= R || W.flat(__ldg(C.idx + p), p) >= x;
    const unsigned m = __ballot_sync(0xffffffffu, ge);
    if (m == 0) {
      L = L + 31 * step + 1;
    } else {
      const int f = __ffs(m) - 1;
      if (f == 0) {
        R = L;
      } else {
        const long long nr = L + f * step;
        L = L + (long long)(f - 1) * step + 1;
        if (nr < R) R = nr;
      }
    }
  }
  const long long p = L + lane;
  const bool ge = p >= R || W.flat(__ldg(C.idx + p), p) >= x;
  const unsigned m = __ballot_sync(0xffffffffu, ge);
  return m ? L + __ffs(m) - 1 : R;
}

__global__ void dm_range_kernel(const __grid_constant__ ContribTable cs, long long a, long long b,
                                long long* __restrict__ ranges) {
  const int c = blockIdx.x;
  const Contrib& C = cs.c[c];
  long long lo, hi;
  if (C.dense) {
    lo = a < C.count ? a : C.count;
    hi = b < C.count ? b : C.count;
  } else {
    Windows W;
    W.load(C.win);
    lo = warp_lower_bound(C, W, a);
    hi = warp_lower_bound(C, W, b);
  }
  if (threadIdx.x == 0) {
    ranges[2 * c] = lo;
    ranges[2 * c + 1] = hi;
  }
}

__device__ __forceinline__ void last_block_release(unsigned* blocks_local, unsigned long long* counter) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned total = gridDim.x * gridDim.y;
    if (atomicAdd(blocks_local, 1u) == total - 1) {
      *blocks_local = 0u;
      __threadfence_system();
      red_release_sys_add_u64(counter, 1ull);
    }
  }
}

// Rank 0's final check that every node's slice landed (the host has already seen every node's completion,
// so this returns at once unless a slice went missing; bounded either way).
__global__ void dm_wait_kernel(const unsigned long long* counter, unsigned long long target, int site,
                               unsigned long long bound_ns) {
  if (threadIdx.x == 0) wait_ge_u64(counter, target, site, bound_ns);
}

// Coefficients of the attempt (this node's control buffer, written by the host on the same stream).
__device__ __forceinline__ void dm_load_coefs(const float* coefs, int n, float* sh_coef) {
  if (threadIdx.x < n) sh_coef[threadIdx.x] = coefs[threadIdx.x];
  __syncthreads();
}

__global__ void dm_apply_dense_kernel(const __grid_constant__ ContribTable cs, int n, long long a4, long long b4,
                                      const float* coefs, float* __restrict__ theta) {
  __shared__ float shc[MAX_CONTRIB];
  dm_load_coefs(coefs, n, shc);
  for (long long i = a4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < b4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < n; ++c) {
      const Contrib& C = cs.c[c];
      const float k = shc[c];
      if (!C.dense || k == 0.f || 4 * i >= C.count) continue;
      const float4 v = __ldg(reinterpret_cast<const float4*>(C.val) + i);
      acc.x += k * v.x;
      acc.y += k * v.y;
      acc.z += k * v.z;
      acc.w += k * v.w;
    }
    float4 t = reinterpret_cast<float4*>(theta)[i];
    t.x += acc.x;
    t.y += acc.y;
    t.z += acc.z;
    t.w += acc.w;
    reinterpret_cast<float4*>(theta)[i] = t;
  }
}

__global__ void dm_apply_sparse_kernel(const __grid_constant__ ContribTable cs, int n,
                                       const long long* __restrict__ ranges, const float* coefs,
                                       float* __restrict__ theta) {
  __shared__ float shc[MAX_CONTRIB];
  dm_load_coefs(coefs, n, shc);
  const int c = blockIdx.y;
  const Contrib& C = cs.c[c];
  const float k = shc[c];
  if (C.dense || k == 0.f) return;
  Windows W;
  W.load(C.win);
  const long long lo = ranges[2 * c], hi = ranges[2 * c + 1];
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = lo + blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < hi; i0 += stride * MUNR) {
    int j[MUNR];
    float v[MUNR];
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      j[u] = i < hi ? __ldg(C.idx + i) : -1;
      v[u] = i < hi ? contrib_value(C, i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < MUNR; ++u)
      if (j[u] >= 0) atomicAdd(theta + W.flat(j[u], i0 + u * stride), v[u] * k);
  }
}

__global__ void dm_broadcast_kernel(const float* __restrict__ theta, long long a4, long long b4, float* mc32, Dests d,
                                    unsigned long long* done_dst, unsigned* blocks_local) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = a4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < b4; i0 += stride * MUNR) {
    float4 t[MUNR];
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      if (i < b4) t[u] = reinterpret_cast<const float4*>(theta)[i];
    }
#pragma unroll
    for (int u = 0; u < MUNR; ++u) {
      const long long i = i0 + u * stride;
      if (i < b4) store_dests(mc32, d, theta, i, t[u]);
    }
  }
  last_block_release(blocks_local, done_dst);
}

// ───── fused tile merge: atomic-free apply + broadcast of one slice (alternative to dm_apply_* + dm_broadcast) ─────
// The slice [a, b) is cut into tiles of DM_TILE elements. dm_tile_bounds_kernel finds, for every sparse
// member payload, the position where each tile's entries start (bounds[c * (ntiles + 1) + t]).
// dm_tile_apply_kernel then gives every tile to one CTA: the CTA loads its tile of the checkpoint and of the
// dense members into registers, sums the entries of all sparse members that fall in the tile into shared
// memory (one flat loop over the concatenation of the members' entry ranges, so every member's loads are in
// flight together; shared atomics only), adds the sum to the checkpoint once and writes the tile to every
// node. Every index is range-checked, so malformed bounds can only skip work.
constexpr int DM_TILE = 4096;
constexpr int DM_TILE_THREADS = 256;
constexpr int DM_TILE_R = DM_TILE / 4 / DM_TILE_THREADS;  // float4s of the tile per thread
constexpr int DM_UNR = 8;

// bounds[c * (ntiles + 1) + t] = the first position of member c's slice range [lo, hi) whose flat index is at
// least a + t * DM_TILE (hi for t = ntiles): one binary search per (member, tile boundary), all independent.
__global__ void dm_tile_bounds_kernel(const __grid_constant__ ContribTable cs, const long long* __restrict__ ranges,
                                      long long a, long long ntiles, long long* __restrict__ bounds) {
  const int c = blockIdx.y;
  const Contrib& C = cs.c[c];
  if (C.dense) return;  // dense members are read directly by tile
  long long* bc = bounds + (long long)c * (ntiles + 1);
  const long long lo0 = ranges[2 * c], hi0 = ranges[2 * c + 1];
  Windows W;
  W.load(C.win);
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t <= ntiles;
       t += (long long)gridDim.x * blockDim.x) {
    const long long key = a + t * DM_TILE;
    long long lo = lo0, hi = hi0 > lo0 ? hi0 : lo0;
    if (t == ntiles) lo = hi;
    while (lo < hi) {
      const long long mid = lo + ((hi - lo) >> 1);
      if (W.flat(__ldg(C.idx + mid), mid) < key) lo = mid + 1;
      else hi = mid;
    }
    bc[t] = lo;
  }
}

__global__ void __launch_bounds__(DM_TILE_THREADS) dm_tile_apply_kernel(
    const __grid_constant__ ContribTable cs, int n, const long long* __restrict__ ranges,
    const long long* __restrict__ bounds, long long a, long long b, long long ntiles, const float* __restrict__ coefs,
    float* theta, float* mc32, Dests d, unsigned long long* done_dst, unsigned* blocks_local) {
  __shared__ __align__(16) float tile[DM_TILE];
  __shared__ long long sh_p0[MAX_CONTRIB], sh_nxt[MAX_CONTRIB];  // first entry in the tile; next window start
  __shared__ int sh_pre[MAX_CONTRIB + 1];                        // prefix of the members' entry counts
  __shared__ int sh_cnt[MAX_CONTRIB];
  __shared__ long long sh_w0[MAX_CONTRIB];                       // window offset (<< 31) at the first entry
  __shared__ float shc[MAX_CONTRIB];
  const int tid = threadIdx.x;
  const long long t = blockIdx.x;
  const long long t0 = a + t * DM_TILE;
  const long long len4 = ((b - t0) < DM_TILE ? (b - t0) : DM_TILE) / 4;  // a, b, DM_TILE multiples of 4
  const long long len = 4 * len4;
  // (1) each member's entry range in this tile; the sparse sum starts at zero
  if (tid < n) {
    const Contrib& C = cs.c[tid];
    const float k = coefs[tid];
    shc[tid] = k;
    long long p0 = 0, nxt = 0x7fffffffffffffffLL, w0 = 0;
    int cnt = 0;
    if (!C.dense && k != 0.f && t < ntiles) {
      const long long lo = ranges[2 * tid], hi = ranges[2 * tid + 1];
      const long long* bc = bounds + (long long)tid * (ntiles + 1);
      long long q0 = bc[t], q1 = bc[t + 1];
      q0 = q0 < lo ? lo : (q0 > hi ? hi : q0);
      q1 = q1 < q0 ? q0 : (q1 > hi ? hi : q1);
      if (q1 - q0 > DM_TILE) q1 = q0 + DM_TILE;  // a tile holds at most DM_TILE distinct indices
      p0 = q0;
      cnt = (int)(q1 - q0);
      if (C.win) {
        for (int w = 1; w < 8; ++w) {
          const long long s = __ldg(C.win + w);
          w0 += (p0 >= s);
          if (s > p0 && s < nxt) nxt = s;
        }
      }
    }
    sh_p0[tid] = p0;
    sh_nxt[tid] = nxt;
    sh_w0[tid] = w0 << 31;
    sh_cnt[tid] = cnt;
  }
  float4* tile4 = reinterpret_cast<float4*>(tile);
  for (int i4 = tid; i4 < DM_TILE / 4; i4 += DM_TILE_THREADS) tile4[i4] = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  // (2) this thread's part of the checkpoint tile plus the dense members, in registers
  float4 th[DM_TILE_R];
#pragma unroll
  for (int r = 0; r < DM_TILE_R; ++r) {
    const long long i4 = tid + r * DM_TILE_THREADS;
    th[r] = i4 < len4 ? reinterpret_cast<const float4*>(theta)[t0 / 4 + i4] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int c = 0; c < n; ++c) {
    const Contrib& C = cs.c[c];
    const float k = shc[c];
    if (!C.dense || k == 0.f) continue;
    float4 v[DM_TILE_R];
#pragma unroll
    for (int r = 0; r < DM_TILE_R; ++r) {
      const long long i4 = tid + r * DM_TILE_THREADS;
      v[r] = (i4 < len4 && t0 + 4 * i4 < C.count) ? __ldg(reinterpret_cast<const float4*>(C.val) + t0 / 4 + i4)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < DM_TILE_R; ++r) {
      th[r].x += k * v[r].x;
      th[r].y += k * v[r].y;
      th[r].z += k * v[r].z;
      th[r].w += k * v[r].w;
    }
  }
  if (tid == 0) {
    int acc = 0;
    for (int c = 0; c < n; ++c) {
      sh_pre[c] = acc;
      acc += sh_cnt[c];
    }
    sh_pre[n] = acc;
  }
  __syncthreads();
  // (3) all sparse members' entries of the tile as one flat list
  const int total = sh_pre[n];
  for (int e0 = tid; e0 < total; e0 += DM_TILE_THREADS * DM_UNR) {
    int j[DM_UNR];
    float v[DM_UNR];
#pragma unroll
    for (int u = 0; u < DM_UNR; ++u) {
      const int e = e0 + u * DM_TILE_THREADS;
      j[u] = -1;
      v[u] = 0.f;
      if (e < total) {
        int lo = 0, hi = n;  // sh_pre[lo] <= e < sh_pre[hi]
        while (hi - lo > 1) {
          const int mid = (lo + hi) >> 1;
          if (sh_pre[mid] <= e) lo = mid;
          else hi = mid;
        }
        const Contrib& C = cs.c[lo];
        const long long p = sh_p0[lo] + (e - sh_pre[lo]);
        const long long flat =
            (long long)__ldg(C.idx + p) + sh_w0[lo] + (p >= sh_nxt[lo] ? (1ll << 31) : 0ll);
        const long long jj = flat - t0;
        j[u] = (jj >= 0 && jj < len) ? (int)jj : -1;
        v[u] = shc[lo] * contrib_value(C, p);
      }
    }
#pragma unroll
    for (int u = 0; u < DM_UNR; ++u)
      if (j[u] >= 0) atomicAdd(&tile[j[u]], v[u]);
  }
  __syncthreads();
  // (4) checkpoint update and broadcast of the tile
#pragma unroll
  for (int r = 0; r < DM_TILE_R; ++r) {
    const long long i4 = tid + r * DM_TILE_THREADS;
    if (i4 < len4) {
      const float4 s = tile4[i4];
      float4 o = th[r];
      o.x += s.x;
      o.y += s.y;
      o.z += s.z;
      o.w += s.w;
      reinterpret_cast<float4*>(theta)[t0 / 4 + i4] = o;
      store_dests(mc32, d, theta, t0 / 4 + i4, o);
    }
  }
  last_block_release(blocks_local, done_dst);
}

// Node side of a checkpoint swap: master <- stage32, p16 <- stage16 (or cast), snapshot <- master.
// Checkpoint swap. rebase == 0: master = snap = staged fp32, p16 = staged bf16 (or its cast).
// rebase == 1: the steps trained since the last push are carried onto the new checkpoint:
// master = staged + (master - snap), snap = staged.
// ef != nullptr folds the error-feedback residual (the part of this node's delta not transmitted yet,
// in "subtract to apply" convention) into the weights: master -= ef, ef = 0. The next delta then
// carries the residual by itself, so what a node transmits is unchanged while it trains on its own
// full progress. p16 = bf16(master) whenever master differs from the staged checkpoint.
__global__ void swap_in_kernel(const float* __restrict__ s32, const __nv_bfloat16* __restrict__ s16,
                               float* __restrict__ master, __nv_bfloat16* __restrict__ p16, float* __restrict__ snap,
                               float* __restrict__ ef, long long n, int rebase) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 t = reinterpret_cast<const float4*>(s32)[i];
    float4 w = t;
    if (rebase) {
      const float4 m = reinterpret_cast<const float4*>(master)[i];
      const float4 o = reinterpret_cast<const float4*>(snap)[i];
      w = make_float4(t.x + (m.x - o.x), t.y + (m.y - o.y), t.z + (m.z - o.z), t.w + (m.w - o.w));
    }
    if (ef) {
      const float4 e = reinterpret_cast<const float4*>(ef)[i];
      w = make_float4(w.x - e.x, w.y - e.y, w.z - e.z, w.w - e.w);
      reinterpret_cast<float4*>(ef)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    reinterpret_cast<float4*>(master)[i] = w;
    if (snap) reinterpret_cast<float4*>(snap)[i] = t;
    if (s16 && !rebase && !ef) {
      reinterpret_cast<uint2*>(p16)[i] = reinterpret_cast<const uint2*>(s16)[i];
    } else {
      uint2 h;
      h.x = pack_bf16(w.x, w.y);
      h.y = pack_bf16(w.z, w.w);
      reinterpret_cast<uint2*>(p16)[i] = h;
    }
  }
}

int grid_cap(long long work, int th, int cap) {
  long long b = (work + th - 1) / th;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

DT_API long long dt_merge_contrib_bytes() { return (long long)sizeof(Contrib); }

// contribs: device array of `n` Contrib descriptors (layout: see struct; sizeof from dt_merge_contrib_bytes).
// `contribs`: HOST array of n packed Contrib records (n <= 64), copied into the launch parameters.
DT_API int dt_merge_prepass(const void* contribs, int n, long long max_count, double* stats, cudaStream_t st) {
  if (n <= 0) return 0;
  if (n > MAX_CONTRIB) return -13;
  DT_CUDA_RET(cudaMemsetAsync(stats, 0, sizeof(double) * 3 * n, st));
  dim3 grid(grid_cap(max_count, 256, 148 * 2), n);
  ContribTable tab;
  memcpy(tab.c, contribs, sizeof(Contrib) * n);
  prepass_kernel<<<grid, 256, 0, st>>>(tab, n, stats);
  return (int)cudaGetLastError();
}

DT_API int dt_merge_accumulate(const void* contribs, int n, long long max_count, float* acc, cudaStream_t st) {
  if (n <= 0) return 0;
  if (n > MAX_CONTRIB) return -13;
  dim3 grid(grid_cap(max_count, 256, 148 * 4), n);
  ContribTable tab;
  memcpy(tab.c, contribs, sizeof(Contrib) * n);
  accumulate_kernel<<<grid, 256, 0, st>>>(tab, n, acc);
  return (int)cudaGetLastError();
}

// stage32: host array of n_dest device pointers (peer-mapped), used when mc32 is null.
static int make_dests(Dests& d, void* mc32, void* const* stage32, int n_dest) {
  if (n_dest > 8) return -11;
  d = Dests{};
  d.n = mc32 ? 0 : n_dest;
  if (!mc32 && (!stage32 || n_dest <= 0)) return -12;
  for (int r = 0; r < d.n; ++r) d.stage32[r] = reinterpret_cast<float*>(stage32[r]);
  return 0;
}

DT_API int dt_merge_apply_broadcast(float* theta, float* vel, float* acc, long long n, float lr, float mu, void* mc32,
                                    void* const* stage32, int n_dest, cudaStream_t st) {
  if (n % 4) return -10;
  Dests d;
  if (int e = make_dests(d, mc32, stage32, n_dest)) return e;
  apply_broadcast_kernel<<<grid_cap(n / 4, 256, 148 * 8), 256, 0, st>>>(theta, vel, acc, n, lr, mu,
                                                                        reinterpret_cast<float*>(mc32), d);
  return (int)cudaGetLastError();
}

DT_API int dt_merge_broadcast(const float* theta, long long n, void* mc32, void* const* stage32, int n_dest,
                              cudaStream_t st) {
  if (n % 4) return -10;
  Dests d;
  if (int e = make_dests(d, mc32, stage32, n_dest)) return e;
  broadcast_kernel<<<grid_cap(n / 4 / MUNR, 256, 148 * 8), 256, 0, st>>>(theta, n, reinterpret_cast<float*>(mc32), d);
  return (int)cudaGetLastError();
}

DT_API int dt_swap_in(const float* s32, const void* s16, float* master, void* p16, float* snap, float* ef,
                      long long n, int rebase, cudaStream_t st) {
  if (n % 4) return -10;
  if ((rebase || ef) && !snap) return -11;
  swap_in_kernel<<<grid_cap(n / 4, 256, 148 * 8), 256, 0, st>>>(s32, reinterpret_cast<const __nv_bfloat16*>(s16),
                                                               master, reinterpret_cast<__nv_bfloat16*>(p16), snap, ef,
                                                               n, rebase);
  return (int)cudaGetLastError();
}

// ───────────────────────────── distributed merge entry points ─────────────────────────────
// `contribs`: host table of n packed Contrib records (as dt_merge_prepass). Ranges scratch: 2*n int64.
DT_API int dt_dm_range(const void* contribs, int n, long long a, long long b, long long* ranges, cudaStream_t st) {
  if (n <= 0) return 0;
  if (n > MAX_CONTRIB) return -13;
  ContribTable tab;
  memcpy(tab.c, contribs, sizeof(Contrib) * n);
  dm_range_kernel<<<n, 32, 0, st>>>(tab, a, b, ranges);
  return (int)cudaGetLastError();
}

DT_API int dt_dm_wait(const unsigned long long* counter, unsigned long long target, int site,
                      unsigned long long bound_ns, cudaStream_t st) {
  dm_wait_kernel<<<1, 32, 0, st>>>(counter, target, site, bound_ns);
  return (int)cudaGetLastError();
}

// Adds the weighted members into theta[a, b) (a, b multiples of 4); coefs: this node's device copy.
DT_API int dt_dm_apply(const void* contribs, int n, long long max_len, const long long* ranges, long long a, long long b,
                       const float* coefs, float* theta, int has_dense, int has_sparse, cudaStream_t st) {
  if (n <= 0 || n > MAX_CONTRIB) return -13;
  if ((a | b) & 3) return -10;
  ContribTable tab;
  memcpy(tab.c, contribs, sizeof(Contrib) * n);
  if (has_dense && b > a)
    dm_apply_dense_kernel<<<grid_cap((b - a) / 4, 256, 148 * 4), 256, 0, st>>>(tab, n, a / 4, b / 4, coefs, theta);
  if (has_sparse) {
    dim3 grid(grid_cap(max_len / MUNR + 1, 256, 148 * 4), n);
    dm_apply_sparse_kernel<<<grid, 256, 0, st>>>(tab, n, ranges, coefs, theta);
  }
  return (int)cudaGetLastError();
}

DT_API int dt_dm_broadcast(const float* theta, long long a, long long b, void* mc32, void* const* stage32, int n_dest,
                           unsigned long long* done_dst, unsigned* blocks_local, cudaStream_t st) {
  if ((a | b) & 3) return -10;
  Dests d;
  if (int e = make_dests(d, mc32, stage32, n_dest)) return e;
  const long long n4 = (b - a) / 4;
  dm_broadcast_kernel<<<grid_cap(n4 / MUNR + 1, 256, 148 * 4), 256, 0, st>>>(theta, a / 4, b / 4,
                                                                             reinterpret_cast<float*>(mc32), d,
                                                                             done_dst, blocks_local);
  return (int)cudaGetLastError();
}

// Fused alternative to dt_dm_apply + dt_dm_broadcast for a slice [a, b) (multiples of 4): tile bounds per
// sparse member into `bounds` (n * (ceil((b - a) / dt_dm_tile_elems()) + 1) int64, device), then one CTA
// per tile.
DT_API long long dt_dm_tile_elems() { return DM_TILE; }

DT_API int dt_dm_fused(const void* contribs, int n, const long long* ranges, long long* bounds, long long a,
                       long long b, const float* coefs, float* theta, void* mc32, void* const* stage32,
                       int n_dest, unsigned long long* done_dst, unsigned* blocks_local, cudaStream_t st) {
  if (n <= 0 || n > MAX_CONTRIB) return -13;
  if ((a | b) & 3) return -10;
  Dests d;
  if (int e = make_dests(d, mc32, stage32, n_dest)) return e;
  ContribTable tab;
  memcpy(tab.c, contribs, sizeof(Contrib) * n);
  const long long ntiles = (b - a + DM_TILE - 1) / DM_TILE;
  if (ntiles > 0) {
    dim3 g1(grid_cap(ntiles + 1, 256, 148 * 8), n);
    dm_tile_bounds_kernel<<<g1, 256, 0, st>>>(tab, ranges, a, ntiles, bounds);
    dm_tile_apply_kernel<<<(unsigned)ntiles, DM_TILE_THREADS, 0, st>>>(tab, n, ranges, bounds, a, b, ntiles, coefs,
                                                                     theta, reinterpret_cast<float*>(mc32), d,
                                                                     done_dst, blocks_local);
  } else {
    // an empty slice still reports completion
    dm_broadcast_kernel<<<1, 32, 0, st>>>(theta, a / 4, b / 4, reinterpret_cast<float*>(mc32), d, done_dst,
                                          blocks_local);
  }
  return (int)cudaGetLastError();
}
