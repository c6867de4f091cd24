// Fused delta compression for one node push, over the flat fp32 parameter buffer:
//
//   d   = snap - master + ef            (outer delta with error feedback; reference training.rs:50-61,
//                                        compression.rs:68-79)
//   snap= master                        (next round starts here)
//   per tensor: k_s from the (adaptive, norm-proportional) budget   (compression.rs:128-159)
//   keep the k_s largest |d| of each tensor, ties by ascending index (the reference's stable sort,
//   compression.rs:162-167), emitted as ascending flat indices
//   ef  = d with the kept entries zeroed  (residual of sparsification, compression.rs:82-88)
//   values quantized to int8 with one absmax/127 fp32 scale per block of 256 kept values
//   (per-tensor scale of the reference = a block spanning the whole tensor), round half away from zero
//
// Exact top-k uses a 3-level radix select on the IEEE bit pattern of |d| (bits 30..19, 18..7, 6..0),
// with per-tensor histograms; the ordered compaction is a chunk-count / scan / write pass, so the
// whole pipeline is a fixed number of linear passes with no sort.
//
// Launch split: dt_compress_begin (pass A) goes on the training stream because it reads the live
// master weights; everything after it only touches `ef` and the payload and runs on a side stream.
#include "common.cuh"

namespace {

constexpr int NB1 = 4096, NB2 = 4096, NB3 = 128;
constexpr int SH1 = 19, SH2 = 7;
constexpr int TPB = 256;
constexpr int UNR = 4;  // elements per thread per loop iteration in the streaming passes

struct SegState {
  double sumsq;      // sum of d^2 over the segment
  double kept_sq;    // sum of kept d^2
  long long len;
  long long k;       // elements to keep
  unsigned prefix;   // resolved key prefix
  long long krem;    // elements still to take inside the current prefix bin
  unsigned tau;      // threshold key
  long long take_eq; // elements with key == tau to keep (by index order)
  long long eq_base; // scan scratch: global count of key == tau entries before the segment's first chunk
  float maxabs;
  int nonfinite;
};

__device__ __forceinline__ unsigned keyof(float v) { return __float_as_uint(v) & 0x7fffffffu; }

// Exclusive block scan of two counters (blockDim.x a multiple of 32, <= 1024); returns the block totals.
__device__ __forceinline__ void block_scan2(long long a, long long b, long long& ea, long long& eb, long long& ta,
                                            long long& tb, long long* sh /* [2][33] */) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  long long ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long xa = __shfl_up_sync(0xffffffffu, ia, o), xb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += xa; ib += xb; }
  }
  if (lane == 31) { sh[wid] = ia; sh[33 + wid] = ib; }
  __syncthreads();
  if (wid == 0) {
    long long va = lane < nw ? sh[lane] : 0, vb = lane < nw ? sh[33 + lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long xa = __shfl_up_sync(0xffffffffu, va, o), xb = __shfl_up_sync(0xffffffffu, vb, o);
      if (lane >= o) { va += xa; vb += xb; }
    }
    if (lane < nw) { sh[lane] = va; sh[33 + lane] = vb; }  // inclusive warp prefixes
  }
  __syncthreads();
  const long long wa = wid ? sh[wid - 1] : 0, wb = wid ? sh[33 + wid - 1] : 0;
  ea = wa + ia - a;
  eb = wb + ib - b;
  ta = sh[nw - 1];
  tb = sh[33 + nw - 1];
  __syncthreads();  // sh may be reused by the caller's next scan
}

// Histogram increment: one shared atomic per element, except when the whole warp falls in one bin (a
// tensor of equal or all-zero deltas), which is counted by one atomic. Measured against aggregating
// every element over the warp (match_any): the typical delta spreads a warp over many 1/16-octave bins,
// so per-element atomics rarely conflict and the aggregation only cost issue slots (pass A + level 2 of
// 100.7 M elements: 0.32 ms less at top-k 1 %). Every lane of the warp must call it.
__device__ __forceinline__ void hist_add(unsigned* h, unsigned bin, bool valid) {
  const unsigned key = valid ? bin : 0xffffffffu;
  const unsigned k0 = __shfl_sync(0xffffffffu, key, 0);
  if (__all_sync(0xffffffffu, key == k0) && valid) {
    if ((threadIdx.x & 31) == 0) atomicAdd(&h[bin], 32u);
  } else if (valid) {
    atomicAdd(&h[bin], 1u);
  }
}

// float4 group at element i0 (4-aligned) of a chunk ending at e: full vector load, or the valid lanes
// (zeros beyond e).
__device__ __forceinline__ float4 ld4(const float* __restrict__ p, long long i0, long long e) {
  if (i0 + 4 <= e) return *reinterpret_cast<const float4*>(p + i0);
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (i0 < e) v.x = p[i0];
  if (i0 + 1 < e) v.y = p[i0 + 1];
  if (i0 + 2 < e) v.z = p[i0 + 2];
  return v;
}
__device__ __forceinline__ void st4(float* __restrict__ p, long long i0, long long e, float4 v) {
  if (i0 + 4 <= e) {
    *reinterpret_cast<float4*>(p + i0) = v;
  } else {
    if (i0 < e) p[i0] = v.x;
    if (i0 + 1 < e) p[i0 + 1] = v.y;
    if (i0 + 2 < e) p[i0 + 2] = v.z;
  }
}
__device__ __forceinline__ float f4at(const float4& v, int q) { return q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w; }

// Pass A: combined delta, snapshot refresh, per-segment stats, level-1 histogram. Each thread streams
// PV float4 groups of master / snap / ef per step (chunk starts are 4-aligned) and loads the next step's
// groups before it works on the current ones, so loads stay in flight through the histogram updates.
constexpr int PV = 2;
__global__ void __launch_bounds__(TPB) pass_a_kernel(const float* __restrict__ master, float* __restrict__ snap,
                                                     float* __restrict__ ef, const int* __restrict__ cseg,
                                                     const long long* __restrict__ cstart,
                                                     const long long* __restrict__ cend, SegState* seg,
                                                     unsigned* __restrict__ hist1, int use_ef) {
  __shared__ unsigned h[NB1];
  __shared__ float shs[32];
  for (int i = threadIdx.x; i < NB1; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int c = blockIdx.x, s = cseg[c];
  float ss = 0.f, mx = 0.f;
  int nf = 0;
  const long long e = cend[c];
  constexpr int STEP = TPB * 4 * PV;
  long long i0 = cstart[c];
  float4 m[PV], sv[PV], ev[PV];
  auto load = [&](long long base) {
#pragma unroll
    for (int u = 0; u < PV; ++u) {
      const long long g = base + (long long)(u * TPB + threadIdx.x) * 4;
      m[u] = ld4(master, g, e);
      sv[u] = ld4(snap, g, e);
      ev[u] = use_ef ? ld4(ef, g, e) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  if (i0 < e) load(i0);
  for (; i0 < e; i0 += STEP) {
    float4 cm[PV], cs[PV], ce[PV];
#pragma unroll
    for (int u = 0; u < PV; ++u) { cm[u] = m[u]; cs[u] = sv[u]; ce[u] = ev[u]; }
    if (i0 + STEP < e) load(i0 + STEP);
#pragma unroll
    for (int u = 0; u < PV; ++u) {
      const long long g = i0 + (long long)(u * TPB + threadIdx.x) * 4;
      float4 d;
      d.x = cs[u].x - cm[u].x + ce[u].x;
      d.y = cs[u].y - cm[u].y + ce[u].y;
      d.z = cs[u].z - cm[u].z + ce[u].z;
      d.w = cs[u].w - cm[u].w + ce[u].w;
      if (g < e) {
        st4(snap, g, e, cm[u]);
        st4(ef, g, e, d);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float x = f4at(d, q);
        const bool valid = g + q < e;
        if (valid) {
          if (!isfinite(x)) nf = 1;
          ss += x * x;
          mx = fmaxf(mx, fabsf(x));
        }
        hist_add(h, keyof(x) >> SH1, valid);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NB1; i += blockDim.x)
    if (h[i]) atomicAdd(&hist1[(long long)s * NB1 + i], h[i]);
  float tot = block_sum(ss, shs);
  float m2 = mx;
  for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int*>(&seg[s].maxabs), __float_as_int(m2));
  nf = __syncthreads_or(nf);
  if (threadIdx.x == 0) {
    atomicAdd(&seg[s].sumsq, (double)tot);
    if (nf) seg[s].nonfinite = 1;
  }
}

// Budget per segment (single block): adaptive (norm-proportional) or uniform, reference arithmetic.
__global__ void budget_kernel(SegState* seg, int nseg, float k_fraction, int adaptive) {
  // The norm total is summed in segment order by one thread (the reference's order, so k per tensor is
  // bit-identical to it); the block only stages the square roots in shared memory.
  __shared__ double buf[256];
  __shared__ double tot_norm, tot_len;
  if (threadIdx.x == 0) { tot_norm = 0.0; tot_len = 0.0; }
  for (int base = 0; base < nseg; base += 256) {
    __syncthreads();
    const int s = base + threadIdx.x;
    if (threadIdx.x < 256 && s < nseg) buf[threadIdx.x] = sqrt(seg[s].sumsq);
    __syncthreads();
    if (threadIdx.x == 0) {
      const int cnt = min(256, nseg - base);
      double tn = tot_norm, tl = tot_len;
      for (int i = 0; i < cnt; ++i) {
        tn += buf[i];
        tl += (double)seg[base + i].len;
      }
      tot_norm = tn;
      tot_len = tl;
    }
  }
  __syncthreads();
  const double total_budget = ceil(tot_len * (double)k_fraction);
  for (int s = threadIdx.x; s < nseg; s += blockDim.x) {
    long long len = seg[s].len, k;
    if (adaptive && tot_norm > 0.0) {
      double frac = sqrt(seg[s].sumsq) / tot_norm;
      k = (long long)ceil(total_budget * frac);
      if (k < 1) k = 1;
      if (k > len) k = len;
    } else {
      k = (long long)ceilf((float)len * k_fraction);
      if (k < 1) k = 1;
      if (k > len) k = len;
    }
    seg[s].k = k;
    seg[s].krem = k;
    seg[s].prefix = 0;
  }
}

// Resolve one radix level for every segment: find the bin holding the krem-th largest key. One block per
// segment; thread t owns PER consecutive bins counted from the top, all loaded at once, and a block scan
// of the per-thread sums locates the crossing thread, which walks its own bins.
template <int NB, int NT>
__global__ void __launch_bounds__(NT) select_level_kernel(SegState* seg, int nseg, const unsigned* __restrict__ hist,
                                                          int bits, int last) {
  constexpr int PER = NB / NT;
  __shared__ long long sh[66];
  const int s = blockIdx.x;
  if (s >= nseg) return;
  const unsigned* hs = hist + (long long)s * NB;
  unsigned local[PER];
  long long tsum = 0;
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    local[u] = hs[NB - 1 - (threadIdx.x * PER + u)];
    tsum += local[u];
  }
  long long above, dummy, total, tdummy;
  block_scan2(tsum, 0, above, dummy, total, tdummy, sh);
  const long long need = seg[s].krem;
  int found = -1;
  long long found_above = 0;
  if (above < need && need <= above + tsum) {
    long long acc = above;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      if (found < 0 && acc + local[u] >= need) {
        found = NB - 1 - (threadIdx.x * PER + u);
        found_above = acc;
      }
      acc += local[u];
    }
  } else if (threadIdx.x == 0 && total < need) {  // need exceeds everything (cannot happen when k <= len)
    found = 0;
    found_above = 0;
  }
  if (found >= 0) {
    seg[s].prefix = (seg[s].prefix << bits) | (unsigned)found;
    seg[s].krem = need - found_above;
    if (last) {
      seg[s].tau = seg[s].prefix;
      seg[s].take_eq = seg[s].krem;
    }
  }
}

// Level-2/3 histogram over elements whose higher bits match the resolved prefix.
// `only_if`: run only when *only_if is set (the candidate path overflowed); nullptr = always.
template <int NB, int SHIFT_MATCH, int SHIFT_BIN>
__global__ void hist_level_kernel(const float* __restrict__ ef, const int* __restrict__ cseg,
                                  const long long* __restrict__ cstart, const long long* __restrict__ cend,
                                  const SegState* seg, unsigned* __restrict__ hist, const int* only_if) {
  if (only_if && !*only_if) return;
  __shared__ unsigned h[NB];
  for (int i = threadIdx.x; i < NB; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int c = blockIdx.x, s = cseg[c];
  const unsigned pre = seg[s].prefix;
  bool any = false;
  const long long e = cend[c];
  for (long long i0 = cstart[c]; i0 < e; i0 += (long long)blockDim.x * UNR) {
    unsigned k[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const long long i = i0 + u * blockDim.x + threadIdx.x;
      k[u] = i < e ? keyof(ef[i]) : 0xffffffffu;  // never matches a prefix (bit 31 set)
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const bool hit = (k[u] >> SHIFT_MATCH) == pre;
      any |= hit;
      if (__any_sync(0xffffffffu, hit)) hist_add(h, (k[u] >> SHIFT_BIN) & (NB - 1), hit);
    }
  }
  any = __syncthreads_or(any);
  if (!any) return;
  for (int i = threadIdx.x; i < NB; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[(long long)s * NB + i], h[i]);
}

// Level-2 pass that also keeps the level-1 boundary bin's keys: every element whose top 12 key bits
// equal the segment's level-1 prefix is counted into the level-2 histogram and its key is staged in
// shared memory, then written to the chunk's candidate slot (CAND keys); the chunk's count of keys above
// the boundary bin goes to gt[c]. The levels after this one (and the per-chunk counts the compaction
// needs) then read the candidates instead of the whole buffer. A chunk with more than CAND candidates
// sets *overflow and the full-buffer passes run instead (bit-identical selection either way).
constexpr int CAND = 1536;
__global__ void __launch_bounds__(TPB) hist2_cand_kernel(const float* __restrict__ ef, const int* __restrict__ cseg,
                                                         const long long* __restrict__ cstart,
                                                         const long long* __restrict__ cend, const SegState* seg,
                                                         unsigned* __restrict__ hist, unsigned* __restrict__ cand,
                                                         int* __restrict__ cand_n, long long* __restrict__ gt,
                                                         int* __restrict__ overflow) {
  __shared__ unsigned h[NB2];
  __shared__ unsigned sc[CAND];
  __shared__ int ns;
  __shared__ unsigned shc[32];
  for (int i = threadIdx.x; i < NB2; i += blockDim.x) h[i] = 0;
  if (threadIdx.x == 0) ns = 0;
  __syncthreads();
  const int c = blockIdx.x, s = cseg[c];
  const unsigned pre = seg[s].prefix;
  const int lane = threadIdx.x & 31;
  unsigned above = 0;
  const long long e = cend[c];
  constexpr int V = 4;  // float4 groups per thread per step (16 elements)
  constexpr int STEP = TPB * 4 * V;
  long long i0 = cstart[c];
  float4 v[V];
  auto load = [&](long long base) {
#pragma unroll
    for (int u = 0; u < V; ++u) v[u] = ld4(ef, base + (long long)(u * TPB + threadIdx.x) * 4, e);
  };
  if (i0 < e) load(i0);
  for (; i0 < e; i0 += STEP) {
    float4 cur[V];
#pragma unroll
    for (int u = 0; u < V; ++u) cur[u] = v[u];
    if (i0 + STEP < e) load(i0 + STEP);
#pragma unroll
    for (int u = 0; u < V; ++u) {
      const long long g = i0 + (long long)(u * TPB + threadIdx.x) * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const unsigned k = keyof(f4at(cur[u], q));
        const bool valid = g + q < e;
        const bool hit = valid && (k >> SH1) == pre;
        above += valid && (k >> SH1) > pre;
        const unsigned hm = __ballot_sync(0xffffffffu, hit);
        if (hm) {
          hist_add(h, (k >> SH2) & (NB2 - 1), hit);
          int base = 0;
          if (lane == 0) base = atomicAdd(&ns, __popc(hm));
          base = __shfl_sync(0xffffffffu, base, 0);
          const int slot = base + __popc(hm & ((1u << lane) - 1));
          if (hit && slot < CAND) sc[slot] = k;
        }
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NB2; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[(long long)s * NB2 + i], h[i]);
  const int n = ns;
  if (n > CAND) {
    if (threadIdx.x == 0) *overflow = 1;
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) cand[(long long)c * CAND + i] = sc[i];
  }
  for (int o = 16; o > 0; o >>= 1) above += __shfl_xor_sync(0xffffffffu, above, o);
  if (lane == 0) shc[threadIdx.x >> 5] = above;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += shc[w];
    gt[c] = t;
    cand_n[c] = n;
  }
}

// Level 3 from the candidates (one block per chunk): keys matching the segment's 24-bit prefix go into the
// segment's 128-bin histogram and the chunk's own 128-bin histogram (h3c); candidates above the prefix add
// to the chunk's count of keys above (gt). Does nothing when a chunk overflowed its candidate slot.
__global__ void __launch_bounds__(128) hist3_cand_kernel(const int* __restrict__ cseg, const SegState* seg,
                                                         const unsigned* __restrict__ cand,
                                                         const int* __restrict__ cand_n, const int* overflow,
                                                         unsigned* __restrict__ hist3, unsigned* __restrict__ h3c,
                                                         long long* __restrict__ gt) {
  if (*overflow) return;
  __shared__ unsigned h[NB3];
  __shared__ unsigned ab;
  h[threadIdx.x] = 0;
  if (threadIdx.x == 0) ab = 0;
  __syncthreads();
  const int c = blockIdx.x, s = cseg[c], n = cand_n[c];
  const unsigned pre = seg[s].prefix;
  unsigned above = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned k = cand[(long long)c * CAND + i];
    if ((k >> SH2) == pre) atomicAdd(&h[k & (NB3 - 1)], 1u);
    above += (k >> SH2) > pre;
  }
  for (int o = 16; o > 0; o >>= 1) above += __shfl_xor_sync(0xffffffffu, above, o);
  if ((threadIdx.x & 31) == 0 && above) atomicAdd(&ab, above);
  __syncthreads();
  const unsigned v = h[threadIdx.x];
  h3c[(long long)c * NB3 + threadIdx.x] = v;
  if (v) atomicAdd(&hist3[(long long)s * NB3 + threadIdx.x], v);
  if (threadIdx.x == 0) gt[c] += ab;
}

// Per chunk, from its level-3 histogram once tau is known: keys == tau, and the keys above tau inside the
// 24-bit prefix bin added to gt. One warp per chunk.
__global__ void chunk_counts_kernel(const int* __restrict__ cseg, int nchunks, const SegState* seg,
                                    const unsigned* __restrict__ h3c, const int* overflow,
                                    long long* __restrict__ gt, long long* __restrict__ eq) {
  if (*overflow) return;
  const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (c >= nchunks) return;
  const unsigned lo = seg[cseg[c]].tau & (NB3 - 1);
  unsigned a = 0, q = 0;
#pragma unroll
  for (int u = 0; u < NB3 / 32; ++u) {
    const int b = u * 32 + lane;
    const unsigned v = h3c[(long long)c * NB3 + b];
    a += (unsigned)b > lo ? v : 0u;
    q += (unsigned)b == lo ? v : 0u;
  }
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  if (lane == 0) {
    gt[c] += a;
    eq[c] = q;
  }
}

// Per chunk: count of keys > tau and == tau (full pass; the candidate path's fallback).
__global__ void count_kernel(const float* __restrict__ ef, const int* __restrict__ cseg,
                             const long long* __restrict__ cstart, const long long* __restrict__ cend,
                             const SegState* seg, long long* __restrict__ cnt_gt, long long* __restrict__ cnt_eq,
                             const int* only_if) {
  if (only_if && !*only_if) return;
  const int c = blockIdx.x, s = cseg[c];
  const unsigned tau = seg[s].tau;
  unsigned gt = 0, eq = 0;
  const long long e = cend[c];
  for (long long i0 = cstart[c]; i0 < e; i0 += (long long)blockDim.x * UNR) {
    unsigned k[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const long long i = i0 + u * blockDim.x + threadIdx.x;
      k[u] = i < e ? keyof(ef[i]) : 0u;
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const long long i = i0 + u * blockDim.x + threadIdx.x;
      gt += (i < e) && (k[u] > tau);
      eq += (i < e) && (k[u] == tau);
    }
  }
  __shared__ unsigned a[32], b[32];
  for (int o = 16; o > 0; o >>= 1) {
    gt += __shfl_xor_sync(0xffffffffu, gt, o);
    eq += __shfl_xor_sync(0xffffffffu, eq, o);
  }
  if ((threadIdx.x & 31) == 0) { a[threadIdx.x >> 5] = gt; b[threadIdx.x >> 5] = eq; }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned tg = 0, te = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { tg += a[w]; te += b[w]; }
    cnt_gt[c] = tg;
    cnt_eq[c] = te;
  }
}

// Single block (1024 threads, each owning a contiguous run of chunks): eq quota per chunk (ties taken in
// index order within each segment) and global output offsets, as two block scans.
__global__ void __launch_bounds__(1024) scan_kernel(const int* __restrict__ cseg, int nchunks, SegState* seg,
                                                    const long long* __restrict__ cnt_gt,
                                                    const long long* __restrict__ cnt_eq,
                                                    long long* __restrict__ eq_take, long long* __restrict__ out_off,
                                                    long long* __restrict__ total) {
  __shared__ long long sh[66];
  const int per = (nchunks + blockDim.x - 1) / blockDim.x;
  const int c0 = min((int)threadIdx.x * per, nchunks), c1 = min(c0 + per, nchunks);
  // 1) global exclusive prefix of the eq counts; the prefix at a segment's first chunk is its base
  long long eqs = 0;
  for (int c = c0; c < c1; ++c) eqs += cnt_eq[c];
  long long ex, dummy, tot_eq, tot_dummy;
  block_scan2(eqs, 0, ex, dummy, tot_eq, tot_dummy, sh);
  for (int c = c0; c < c1; ++c) {
    eq_take[c] = ex;  // eq entries of all chunks before c (temporary)
    if (c == 0 || cseg[c - 1] != cseg[c]) seg[cseg[c]].eq_base = ex;
    ex += cnt_eq[c];
  }
  __syncthreads();
  // 2) eq entries this chunk may take, then the global exclusive prefix of kept entries
  long long kept = 0;
  for (int c = c0; c < c1; ++c) {
    const int s = cseg[c];
    long long q = seg[s].take_eq - (eq_take[c] - seg[s].eq_base);
    q = q < 0 ? 0 : (q > cnt_eq[c] ? cnt_eq[c] : q);
    eq_take[c] = q;
    kept += cnt_gt[c] + q;
  }
  long long off, tot;
  block_scan2(kept, 0, off, dummy, tot, tot_dummy, sh);
  for (int c = c0; c < c1; ++c) {
    out_off[c] = off;
    off += cnt_gt[c] + eq_take[c];
  }
  if (threadIdx.x == 0) *total = tot;
}

// Kept indices are stored as 32-bit offsets within 2^31-element windows of the flat buffer (chunks never
// straddle a window boundary); the payload records the position where each window's entries start, so a
// reader adds (window << 31). Buffers below 2^31 elements have one window and plain indices.
constexpr long long kWindowMask = (1LL << 31) - 1;
constexpr int kMaxWindows = 8;

__global__ void window_kernel(const long long* __restrict__ off, const long long* __restrict__ total,
                              const int* __restrict__ win_chunk, int nwin, int nchunks, long long* __restrict__ out) {
  const int k = threadIdx.x;
  if (k >= kMaxWindows) return;
  long long v = 0x7fffffffffffffffLL;  // no such window
  if (k == 0) {
    v = 0;
  } else if (k < nwin) {
    const int c = win_chunk[k];
    v = c < nchunks ? off[c] : *total;
  }
  out[k] = v;
}

// Ordered compaction: writes (index, value) of kept entries in ascending index order, zeroes them in ef.
// A round covers CG x 1024 elements: thread t loads the float4 groups t, t + 256, ... (coalesced), so
// the round's index order is (group, thread, lane of the float4). The per-group counts of keys > tau and
// == tau are packed as 16-bit fields (a field's block total is at most 1024) into two 64-bit words, and
// one block scan of the pair gives every thread its output position and its share of the chunk's tie
// quota for all CG groups at once.
__device__ __forceinline__ void f4zero(float4& v, int q) {
  if (q == 0) v.x = 0.f;
  else if (q == 1) v.y = 0.f;
  else if (q == 2) v.z = 0.f;
  else v.w = 0.f;
}
__device__ __forceinline__ long long fld(long long w, int j) { return (w >> (16 * j)) & 0xffff; }

constexpr int CG = 4;
__global__ void __launch_bounds__(TPB) compact_kernel(float* __restrict__ ef, const int* __restrict__ cseg,
                                                      const long long* __restrict__ cstart,
                                                      const long long* __restrict__ cend, SegState* seg,
                                                      const long long* __restrict__ eq_take,
                                                      const long long* __restrict__ out_off, int* __restrict__ out_idx,
                                                      float* __restrict__ out_val, long long capacity) {
  __shared__ long long sh[66];
  __shared__ float shs[32];
  const int c = blockIdx.x, s = cseg[c];
  const unsigned tau = seg[s].tau;
  const long long quota = eq_take[c];
  const long long e = cend[c];
  long long base_sel = out_off[c], eq_seen = 0;
  float kept_sq = 0.f;
  constexpr int ROUND = TPB * 4 * CG;
  // the next round's groups are loaded before this round's scan and writes (chunk starts are 4-aligned)
  float4 nxt[CG];
  auto load = [&](long long base) {
#pragma unroll
    for (int j = 0; j < CG; ++j) nxt[j] = ld4(ef, base + (long long)j * (TPB * 4) + threadIdx.x * 4, e);
  };
  if (cstart[c] < e) load(cstart[c]);
  for (long long r0 = cstart[c]; r0 < e; r0 += ROUND) {
    float4 v[CG];
#pragma unroll
    for (int j = 0; j < CG; ++j) v[j] = nxt[j];
    if (r0 + ROUND < e) load(r0 + ROUND);
    unsigned gtm = 0, eqm = 0;  // bit 4 * group + lane of the float4
    long long gpack = 0, epack = 0;
#pragma unroll
    for (int j = 0; j < CG; ++j) {
      const long long i0 = r0 + (long long)j * (TPB * 4) + threadIdx.x * 4;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const unsigned k = keyof(f4at(v[j], q));
        const bool valid = i0 + q < e;
        if (valid && k > tau) gtm |= 1u << (4 * j + q);
        if (valid && k == tau) eqm |= 1u << (4 * j + q);
      }
      gpack |= (long long)__popc((gtm >> (4 * j)) & 15u) << (16 * j);
      epack |= (long long)__popc((eqm >> (4 * j)) & 15u) << (16 * j);
    }
    long long gpre, epre, gtot, etot;
    block_scan2(gpack, epack, gpre, epre, gtot, etot, sh);
    const long long qrem = quota - eq_seen > 0 ? quota - eq_seen : 0;  // ties this chunk may still take
    long long gs = 0, es = 0;  // keys > tau / == tau in the round's earlier groups
#pragma unroll
    for (int j = 0; j < CG; ++j) {
      const long long i0 = r0 + (long long)j * (TPB * 4) + threadIdx.x * 4;
      long long gb = gs + fld(gpre, j), eb = es + fld(epre, j);
      bool any = false;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int bit = 4 * j + q;
        const bool is_gt = (gtm >> bit) & 1u, is_eq = (eqm >> bit) & 1u;
        if (is_gt || (is_eq && eb < qrem)) {
          const long long pos = base_sel + gb + (eb < qrem ? eb : qrem);
          const float x = f4at(v[j], q);
          if (pos < capacity) {
            out_idx[pos] = (int)((i0 + q) & kWindowMask);  // index within its 2^31 window
            out_val[pos] = x;
            kept_sq += x * x;
            f4zero(v[j], q);
            any = true;
          } else {
            // the caller's output arrays are too short: keep the value in error feedback, write nothing
            dt_set_error(DT_ERR_BOUNDS, 710);
          }
        }
        gb += is_gt;
        eb += is_eq;
      }
      if (any) {
        if (i0 + 4 <= e) {
          *reinterpret_cast<float4*>(ef + i0) = v[j];
        } else {
          for (int q = 0; q < 3 && i0 + q < e; ++q) ef[i0 + q] = f4at(v[j], q);
        }
      }
      gs += fld(gtot, j);
      es += fld(etot, j);
    }
    base_sel += gs + (es < qrem ? es : qrem);
    eq_seen += es;
  }
  float t = block_sum(kept_sq, shs);
  if (threadIdx.x == 0) atomicAdd(&seg[s].kept_sq, (double)t);
}

// Per block of `blk` kept values: absmax/127 scale (1 if all zero), round-half-away int8.
// `wire` (3 doubles): statistics of the dequantised values as they go on the wire - sum of squares,
// max |x| (as ordered bits), non-finite blocks - which the coordinator validates and clips on.
// One warp per block (blk a multiple of 32, at most 32 x QV): the values stay in registers between the
// max and the quantisation, reductions are warp shuffles, and the CTA's eight warps add their wire
// statistics once.
constexpr int QV = 16;
__global__ void __launch_bounds__(256) quant_kernel(const float* __restrict__ val, const long long* __restrict__ total,
                                                   long long capacity, int blk, signed char* __restrict__ q,
                                                   float* __restrict__ scales, double* __restrict__ wire) {
  __shared__ float sss[8], smx[8];
  __shared__ int snf[8];
  const long long n = *total < capacity ? *total : capacity;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long b = (long long)blockIdx.x * 8 + w;
  const long long s0 = b * blk;
  float ss = 0.f, dmax = 0.f;
  int nf = 0;
  if (s0 < n) {
    const long long e = (s0 + blk < n) ? s0 + blk : n;
    const int per = blk >> 5;
    float x[QV];
    float mx = 0.f;
#pragma unroll
    for (int u = 0; u < QV; ++u) {
      const long long i = s0 + (long long)u * 32 + lane;
      x[u] = (u < per && i < e) ? val[i] : 0.f;
      mx = fmaxf(mx, fabsf(x[u]));
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float scale = mx == 0.f ? 1.f : mx / 127.f;
    if (lane == 0) scales[b] = scale;
#pragma unroll
    for (int u = 0; u < QV; ++u) {
      const long long i = s0 + (long long)u * 32 + lane;
      if (u < per && i < e) {
        float r = roundf(x[u] / scale);
        r = fminf(fmaxf(r, -127.f), 127.f);
        q[i] = (signed char)r;
        const float dq = r * scale;
        ss += dq * dq;
        dmax = fmaxf(dmax, fabsf(dq));
      }
    }
    nf = !isfinite(mx);
  }
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    dmax = fmaxf(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
  }
  if (lane == 0) { sss[w] = ss; smx[w] = dmax; snf[w] = nf; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    float m = 0.f;
    int f = 0;
    for (int i = 0; i < 8; ++i) { t += (double)sss[i]; m = fmaxf(m, smx[i]); f += snf[i]; }
    if (t != 0.0) atomicAdd(wire, t);
    if (m > 0.f) atomicMax(reinterpret_cast<unsigned long long*>(wire + 1), (unsigned long long)__double_as_longlong((double)m));
    if (f) atomicAdd(wire + 2, (double)f);
  }
}

}  // namespace

// ───────────────────────────── host API ─────────────────────────────
// Workspace layout (device, caller-allocated, size from dt_compress_workspace_bytes):
//   SegState[nseg] | hist1[nseg*NB1] | hist2[nseg*NB2] | hist3[nseg*NB3] |
//   cnt_gt[nchunks] | cnt_eq[nchunks] | eq_take[nchunks] | out_off[nchunks] | overflow |
//   total[1] wire[3] (doubles) || cand_n[nchunks] | h3c[nchunks*NB3] | cand[nchunks*CAND]
// Everything before "||" is cleared by dt_compress_begin; the candidate region behind it is always
// written before it is read.
struct WsPtrs {
  SegState* seg;
  unsigned *h1, *h2, *h3;
  long long *gt, *eq, *take, *off;
  int* overflow;
  long long* total;
  int* cand_n;
  unsigned *h3c, *cand;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static size_t ws_zeroed_bytes(int nseg, int nchunks) {
  return align256(sizeof(SegState) * nseg) + align256(4ull * nseg * NB1) + align256(4ull * nseg * NB2) +
         align256(4ull * nseg * NB3) + 4 * align256(8ull * nchunks) + 256 + 256;
}

static WsPtrs carve(void* ws, int nseg, int nchunks) {
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  WsPtrs w;
  w.seg = reinterpret_cast<SegState*>(p); p += align256(sizeof(SegState) * nseg);
  w.h1 = reinterpret_cast<unsigned*>(p); p += align256(sizeof(unsigned) * (size_t)nseg * NB1);
  w.h2 = reinterpret_cast<unsigned*>(p); p += align256(sizeof(unsigned) * (size_t)nseg * NB2);
  w.h3 = reinterpret_cast<unsigned*>(p); p += align256(sizeof(unsigned) * (size_t)nseg * NB3);
  w.gt = reinterpret_cast<long long*>(p); p += align256(8 * (size_t)nchunks);
  w.eq = reinterpret_cast<long long*>(p); p += align256(8 * (size_t)nchunks);
  w.take = reinterpret_cast<long long*>(p); p += align256(8 * (size_t)nchunks);
  w.off = reinterpret_cast<long long*>(p); p += align256(8 * (size_t)nchunks);
  w.overflow = reinterpret_cast<int*>(p); p += 256;
  w.total = reinterpret_cast<long long*>(p); p += 256;
  w.cand_n = reinterpret_cast<int*>(p); p += align256(4ull * nchunks);
  w.h3c = reinterpret_cast<unsigned*>(p); p += align256(4ull * nchunks * NB3);
  w.cand = reinterpret_cast<unsigned*>(p);
  return w;
}

DT_API long long dt_compress_workspace_bytes(int nseg, int nchunks) {
  return (long long)(ws_zeroed_bytes(nseg, nchunks) + align256(4ull * nchunks) + align256(4ull * nchunks * NB3) +
                     align256(4ull * nchunks * CAND));
}

DT_API long long dt_compress_segstate_bytes() { return (long long)sizeof(SegState); }

__global__ void seg_init_kernel(SegState* seg, const long long* __restrict__ seg_len, int nseg) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < nseg; s += gridDim.x * blockDim.x) {
    SegState z = {};
    z.len = seg_len[s];
    seg[s] = z;
  }
}

__global__ void export_stats_kernel(const SegState* seg, int nseg, const long long* total, double* out) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < nseg; s += gridDim.x * blockDim.x) {
    out[s * 6 + 0] = seg[s].sumsq;
    out[s * 6 + 1] = seg[s].kept_sq;
    out[s * 6 + 2] = (double)seg[s].k;
    out[s * 6 + 3] = (double)seg[s].maxabs;
    out[s * 6 + 4] = (double)seg[s].nonfinite;
    out[s * 6 + 5] = (double)seg[s].len;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    out[nseg * 6] = (double)*total;
    const double* wire = reinterpret_cast<const double*>(total + 1);  // quantised pushes only
    out[nseg * 6 + 1] = wire[0];
    out[nseg * 6 + 2] = wire[1];
    out[nseg * 6 + 3] = wire[2];
  }
}

// Pass A (training stream). seg_len: device array of per-segment element counts.
DT_API int dt_compress_begin(const float* master, float* snap, float* ef, const int* cseg, const long long* cstart,
                             const long long* cend, int nchunks, int nseg, const long long* seg_len, void* ws,
                             int use_ef, cudaStream_t st) {
  WsPtrs w = carve(ws, nseg, nchunks);
  DT_CUDA_RET(cudaMemsetAsync(ws, 0, ws_zeroed_bytes(nseg, nchunks), st));
  seg_init_kernel<<<(nseg + 255) / 256, 256, 0, st>>>(w.seg, seg_len, nseg);
  pass_a_kernel<<<nchunks, TPB, 0, st>>>(master, snap, ef, cseg, cstart, cend, w.seg, w.h1, use_ef);
  return (int)cudaGetLastError();
}

// Everything after pass A (side stream). Writes out_idx/out_val (capacity entries) in ascending index
// order, int8 + per-block scales when quant_block > 0, and the kept count into the workspace. An entry
// that would land at or beyond `capacity` is not written (it stays in error feedback) and sets
// DT_ERR_BOUNDS in dt_error_word; the per-tensor budgets sum to at most ceil(n * k_fraction) + nseg.
DT_API int dt_compress_finish(float* ef, const int* cseg, const long long* cstart, const long long* cend, int nchunks,
                              int nseg, void* ws, float k_fraction, int adaptive, int* out_idx, float* out_val,
                              signed char* out_q, float* out_scales, int quant_block, long long capacity,
                              const int* win_chunk, int nwin, long long* out_win, cudaStream_t st) {
  if (nwin > kMaxWindows) return -21;
  if (quant_block > 0 && (quant_block % 32 != 0 || quant_block > 32 * QV)) return -24;
  WsPtrs w = carve(ws, nseg, nchunks);
  budget_kernel<<<1, 256, 0, st>>>(w.seg, nseg, k_fraction, adaptive);
  select_level_kernel<NB1, 256><<<nseg, 256, 0, st>>>(w.seg, nseg, w.h1, 12, 0);
  // level 2 over the whole buffer, keeping the level-1 boundary bin's keys per chunk
  hist2_cand_kernel<<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.h2, w.cand, w.cand_n, w.gt,
                                             w.overflow);
  select_level_kernel<NB2, 256><<<nseg, 256, 0, st>>>(w.seg, nseg, w.h2, 12, 0);
  // level 3 from the candidates; the full pass only when a chunk overflowed its candidate slot
  hist3_cand_kernel<<<nchunks, NB3, 0, st>>>(cseg, w.seg, w.cand, w.cand_n, w.overflow, w.h3, w.h3c, w.gt);
  hist_level_kernel<NB3, SH2, 0><<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.h3, w.overflow);
  select_level_kernel<NB3, 128><<<nseg, 128, 0, st>>>(w.seg, nseg, w.h3, 7, 1);
  // per-chunk counts above / at tau: from the chunk histograms, or a full pass after an overflow
  chunk_counts_kernel<<<(nchunks + 7) / 8, 256, 0, st>>>(cseg, nchunks, w.seg, w.h3c, w.overflow, w.gt, w.eq);
  count_kernel<<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.gt, w.eq, w.overflow);
  scan_kernel<<<1, 1024, 0, st>>>(cseg, nchunks, w.seg, w.gt, w.eq, w.take, w.off, w.total);
  compact_kernel<<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.take, w.off, out_idx, out_val, capacity);
  if (out_win) window_kernel<<<1, 32, 0, st>>>(w.off, w.total, win_chunk, nwin, nchunks, out_win);
  if (quant_block > 0 && out_q) {
    const long long nblk = (capacity + quant_block - 1) / quant_block;
    quant_kernel<<<(unsigned)((nblk + 7) / 8), 256, 0, st>>>(out_val, w.total, capacity, quant_block, out_q,
                                                             out_scales, reinterpret_cast<double*>(w.total + 1));
  }
  return (int)cudaGetLastError();
}

// Raw push (no selection): the whole delta + error feedback formed by pass A leaves as dense fp32 and the
// error-feedback buffer is cleared (nothing is left behind). n: a multiple of 4.
__global__ void raw_kernel(float* __restrict__ ef, float* __restrict__ out, long long n4) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    reinterpret_cast<float4*>(out)[i] = reinterpret_cast<const float4*>(ef)[i];
    reinterpret_cast<float4*>(ef)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

DT_API int dt_compress_raw(float* ef, float* out, long long n, cudaStream_t st) {
  if (n % 4) return -10;
  long long b = (n / 4 + 255) / 256;
  if (b > 148 * 8) b = 148 * 8;
  raw_kernel<<<(unsigned)(b < 1 ? 1 : b), 256, 0, st>>>(ef, out, n / 4);
  return (int)cudaGetLastError();
}

// Per-segment statistics into a device double array: [s*6 + {sumsq, kept_sq, k, maxabs, nonfinite, len}],
// then the total kept count at [nseg*6] and the dequantised wire statistics {sum of squares, max |x|,
// non-finite} at [nseg*6 + 1..3] (zero unless the push was quantised).
DT_API long long dt_compress_stats_len(int nseg) { return 6LL * nseg + 4; }

DT_API int dt_compress_export_stats(void* ws, int nseg, int nchunks, double* out, cudaStream_t st) {
  WsPtrs w = carve(ws, nseg, nchunks);
  export_stats_kernel<<<(nseg + 255) / 256, 256, 0, st>>>(w.seg, nseg, w.total, out);
  return (int)cudaGetLastError();
}

// ───────────────────────────── allocation-free entry point ─────────────────────────────
// dt_compress_noalloc: the same pipeline as dt_compress_begin + dt_compress_finish, for callers that
// cannot allocate device memory themselves (see compress_noalloc.h). Its workspace is the file-scope
// array below; host code never dereferences the array's name (on the host it is only a stand-in
// symbol) - the device address comes from cudaGetSymbolAddress, resolved once per device.
#include "compress_noalloc.h"
#include <mutex>

static __device__ __align__(256) unsigned char g_compress_scratch[DT_COMPRESS_NOALLOC_SCRATCH_BYTES];

namespace {
std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {nullptr};
}  // namespace

DT_API long long dt_compress_noalloc_scratch_bytes() { return (long long)DT_COMPRESS_NOALLOC_SCRATCH_BYTES; }

DT_API long long dt_compress_noalloc_min_capacity(long long n_elems, int nseg, float k_fraction) {
  long long c = (long long)ceil((double)n_elems * (double)k_fraction) + nseg;
  return c < n_elems ? c : n_elems;
}

DT_API int dt_compress_noalloc(const float* master, float* snap, float* ef, const int* cseg, const long long* cstart,
                               const long long* cend, int nchunks, int nseg, const long long* seg_len,
                               long long n_elems, float k_fraction, int adaptive, int* out_idx, float* out_val,
                               signed char* out_q, float* out_scales, int quant_block, long long capacity,
                               double* stats_out, cudaStream_t st) {
  if (nseg <= 0 || nchunks <= 0 || n_elems <= 0 || !(k_fraction > 0.f) || k_fraction > 1.f) return -10;
  // kept indices are 32-bit flat offsets: a buffer of 2^31 elements or more needs the windowed payload
  // of dt_compress_finish (win_chunk / out_win), which this entry point does not produce
  if (n_elems > kWindowMask) return -22;
  if (capacity < dt_compress_noalloc_min_capacity(n_elems, nseg, k_fraction)) return -23;
  if (quant_block > 0 && (quant_block % 32 != 0 || quant_block > 32 * QV)) return -24;
  const long long need = dt_compress_workspace_bytes(nseg, nchunks);
  if (need > (long long)DT_COMPRESS_NOALLOC_SCRATCH_BYTES) return -20;
  int dev = 0;
  DT_CUDA_RET(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return -21;
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_compress_scratch);
      if (e != cudaSuccess) return (int)e;
      g_scratch_ptr[dev] = p;
    }
    ws = g_scratch_ptr[dev];
  }
  // dt_compress_begin clears the workspace's histograms and counters before use
  int rc = dt_compress_begin(master, snap, ef, cseg, cstart, cend, nchunks, nseg, seg_len, ws, 1, st);
  if (rc) return rc;
  // below 2^31 elements there is one index window, so the kept indices are plain flat indices
  rc = dt_compress_finish(ef, cseg, cstart, cend, nchunks, nseg, ws, k_fraction, adaptive, out_idx, out_val, out_q,
                          out_scales, quant_block, capacity, nullptr, 1, nullptr, st);
  if (rc) return rc;
  if (stats_out) return dt_compress_export_stats(ws, nseg, nchunks, stats_out, st);
  return 0;
}
