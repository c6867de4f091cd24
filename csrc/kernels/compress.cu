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

// Histogram increment aggregated over the warp: lanes that hit the same bin are counted by one atomic.
// Deltas of one tensor have similar magnitudes and crowd into a few bins, where per-lane shared atomics
// would serialise 32-fold. Every lane of the warp must call it (inactive lanes with valid = false).
__device__ __forceinline__ void hist_add_warp(unsigned* h, unsigned bin, bool valid) {
  const unsigned key = valid ? bin : 0xffffffffu;
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  if (valid && (threadIdx.x & 31) == (unsigned)(__ffs(peers) - 1)) atomicAdd(&h[bin], (unsigned)__popc(peers));
}

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

// Pass A: combined delta, snapshot refresh, per-segment stats, level-1 histogram.
__global__ void pass_a_kernel(const float* __restrict__ master, float* __restrict__ snap, float* __restrict__ ef,
                              const int* __restrict__ cseg, const long long* __restrict__ cstart,
                              const long long* __restrict__ cend, SegState* seg, unsigned* __restrict__ hist1,
                              int use_ef) {
  __shared__ unsigned h[NB1];
  __shared__ float shs[32];
  for (int i = threadIdx.x; i < NB1; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int c = blockIdx.x, s = cseg[c];
  float ss = 0.f, mx = 0.f;
  int nf = 0;
  const long long e = cend[c];
  // UNR elements per thread per iteration, all loads issued before any use (memory-level parallelism)
  for (long long i0 = cstart[c]; i0 < e; i0 += (long long)blockDim.x * UNR) {
    float m[UNR], sv[UNR], ev[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const long long i = i0 + u * blockDim.x + threadIdx.x;
      const bool valid = i < e;
      m[u] = valid ? master[i] : 0.f;
      sv[u] = valid ? snap[i] : 0.f;
      ev[u] = (valid && use_ef) ? ef[i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const long long i = i0 + u * blockDim.x + threadIdx.x;
      const bool valid = i < e;
      const float d = sv[u] - m[u] + ev[u];
      if (valid) {
        snap[i] = m[u];
        ef[i] = d;
        if (!isfinite(d)) nf = 1;
        ss += d * d;
        mx = fmaxf(mx, fabsf(d));
      }
      hist_add_warp(h, keyof(d) >> SH1, valid);
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
template <int NB, int SHIFT_MATCH, int SHIFT_BIN>
__global__ void hist_level_kernel(const float* __restrict__ ef, const int* __restrict__ cseg,
                                  const long long* __restrict__ cstart, const long long* __restrict__ cend,
                                  const SegState* seg, unsigned* __restrict__ hist) {
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
      if (__any_sync(0xffffffffu, hit)) hist_add_warp(h, (k[u] >> SHIFT_BIN) & (NB - 1), hit);
    }
  }
  any = __syncthreads_or(any);
  if (!any) return;
  for (int i = threadIdx.x; i < NB; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[(long long)s * NB + i], h[i]);
}

// Per chunk: count of keys > tau and == tau.
__global__ void count_kernel(const float* __restrict__ ef, const int* __restrict__ cseg,
                             const long long* __restrict__ cstart, const long long* __restrict__ cend,
                             const SegState* seg, long long* __restrict__ cnt_gt, long long* __restrict__ cnt_eq) {
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
// Each thread owns CR consecutive elements per round; one block scan of (keys > tau, keys == tau) counts
// per round gives every thread its output position and its share of the chunk's eq quota.
constexpr int CR = 16;
__global__ void compact_kernel(float* __restrict__ ef, const int* __restrict__ cseg,
                               const long long* __restrict__ cstart, const long long* __restrict__ cend,
                               SegState* seg, const long long* __restrict__ eq_take,
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
  for (long long r0 = cstart[c]; r0 < e; r0 += (long long)blockDim.x * CR) {
    const long long i0 = r0 + (long long)threadIdx.x * CR;
    float v[CR];
    unsigned gtm = 0, eqm = 0;
#pragma unroll
    for (int j = 0; j < CR; ++j) {
      const long long i = i0 + j;
      v[j] = i < e ? ef[i] : 0.f;
      const unsigned k = keyof(v[j]);
      if (i < e && k > tau) gtm |= 1u << j;
      if (i < e && k == tau) eqm |= 1u << j;
    }
    long long gpre, epre, gtot, etot;
    block_scan2(__popc(gtm), __popc(eqm), gpre, epre, gtot, etot, sh);
    const long long qrem = quota - eq_seen;  // ties this chunk may still take, in index order
    const long long eq_before = qrem <= 0 ? 0 : (epre < qrem ? epre : qrem);
    long long allow = qrem - epre;
    long long pos = base_sel + gpre + eq_before;
#pragma unroll
    for (int j = 0; j < CR; ++j) {
      bool take = (gtm >> j) & 1u;
      if (((eqm >> j) & 1u) && allow > 0) {
        take = true;
        --allow;
      }
      if (take) {
        if (pos < capacity) {
          out_idx[pos] = (int)((i0 + j) & kWindowMask);  // index within its 2^31 window
          out_val[pos] = v[j];
          ef[i0 + j] = 0.f;
          kept_sq += v[j] * v[j];
        } else {
          // the caller's output arrays are too short: keep the value in error feedback, write nothing
          dt_set_error(DT_ERR_BOUNDS, 710);
        }
        ++pos;
      }
    }
    base_sel += gtot + (qrem <= 0 ? 0 : (etot < qrem ? etot : qrem));
    eq_seen += etot;
  }
  float t = block_sum(kept_sq, shs);
  if (threadIdx.x == 0) atomicAdd(&seg[s].kept_sq, (double)t);
}

// Per block of `blk` kept values: absmax/127 scale (1 if all zero), round-half-away int8.
// `wire` (3 doubles): statistics of the dequantised values as they go on the wire - sum of squares,
// max |x| (as ordered bits), non-finite blocks - which the coordinator validates and clips on.
__global__ void quant_kernel(const float* __restrict__ val, const long long* __restrict__ total, long long capacity,
                             int blk, signed char* __restrict__ q, float* __restrict__ scales,
                             double* __restrict__ wire) {
  __shared__ float sh[32];
  const long long n = *total < capacity ? *total : capacity;
  const long long b = blockIdx.x;
  const long long s0 = b * blk;
  if (s0 >= n) return;
  const long long e = (s0 + blk < n) ? s0 + blk : n;
  float mx = 0.f;
  for (long long i = s0 + threadIdx.x; i < e; i += blockDim.x) mx = fmaxf(mx, fabsf(val[i]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) sh[0] = v;
  }
  __syncthreads();
  const float amax = sh[0];
  const float scale = amax == 0.f ? 1.f : amax / 127.f;
  if (threadIdx.x == 0) scales[b] = scale;
  float ss = 0.f, dmax = 0.f;
  for (long long i = s0 + threadIdx.x; i < e; i += blockDim.x) {
    float r = roundf(val[i] / scale);
    r = fminf(fmaxf(r, -127.f), 127.f);
    q[i] = (signed char)r;
    const float dq = r * scale;
    ss += dq * dq;
    dmax = fmaxf(dmax, fabsf(dq));
  }
  __syncthreads();  // sh reused
  const float tss = block_sum(ss, sh);
  for (int o = 16; o > 0; o >>= 1) dmax = fmaxf(dmax, __shfl_xor_sync(0xffffffffu, dmax, o));
  if ((threadIdx.x & 31) == 0 && dmax > 0.f)
    atomicMax(reinterpret_cast<unsigned long long*>(wire + 1), (unsigned long long)__double_as_longlong((double)dmax));
  if (threadIdx.x == 0) {
    atomicAdd(wire, (double)tss);
    if (!isfinite(amax)) atomicAdd(wire + 2, 1.0);
  }
}

}  // namespace

// ───────────────────────────── host API ─────────────────────────────
// Workspace layout (device, caller-allocated, size from dt_compress_workspace_bytes):
//   SegState[nseg] | hist1[nseg*NB1] | hist2[nseg*NB2] | hist3[nseg*NB3] |
//   cnt_gt[nchunks] | cnt_eq[nchunks] | eq_take[nchunks] | out_off[nchunks] | total[1] wire[3] (doubles)
struct WsPtrs {
  SegState* seg;
  unsigned *h1, *h2, *h3;
  long long *gt, *eq, *take, *off, *total;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

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
  w.total = reinterpret_cast<long long*>(p);
  return w;
}

DT_API long long dt_compress_workspace_bytes(int nseg, int nchunks) {
  return (long long)(align256(sizeof(SegState) * nseg) + align256(4ull * nseg * NB1) + align256(4ull * nseg * NB2) +
                     align256(4ull * nseg * NB3) + 4 * align256(8ull * nchunks) + 256);
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
  DT_CUDA_RET(cudaMemsetAsync(ws, 0, (size_t)dt_compress_workspace_bytes(nseg, nchunks), st));
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
  WsPtrs w = carve(ws, nseg, nchunks);
  budget_kernel<<<1, 256, 0, st>>>(w.seg, nseg, k_fraction, adaptive);
  select_level_kernel<NB1, 256><<<nseg, 256, 0, st>>>(w.seg, nseg, w.h1, 12, 0);
  hist_level_kernel<NB2, SH1, SH2><<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.h2);
  select_level_kernel<NB2, 256><<<nseg, 256, 0, st>>>(w.seg, nseg, w.h2, 12, 0);
  hist_level_kernel<NB3, SH2, 0><<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.h3);
  select_level_kernel<NB3, 128><<<nseg, 128, 0, st>>>(w.seg, nseg, w.h3, 7, 1);
  count_kernel<<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.gt, w.eq);
  scan_kernel<<<1, 1024, 0, st>>>(cseg, nchunks, w.seg, w.gt, w.eq, w.take, w.off, w.total);
  compact_kernel<<<nchunks, TPB, 0, st>>>(ef, cseg, cstart, cend, w.seg, w.take, w.off, out_idx, out_val, capacity);
  if (out_win) window_kernel<<<1, 32, 0, st>>>(w.off, w.total, win_chunk, nwin, nchunks, out_win);
  if (quant_block > 0 && out_q) {
    long long nblk = (capacity + quant_block - 1) / quant_block;
    quant_kernel<<<(unsigned)nblk, 256, 0, st>>>(out_val, w.total, capacity, quant_block, out_q, out_scales,
                                                 reinterpret_cast<double*>(w.total + 1));
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
  // dt_compress_begin clears the whole workspace (histograms, counters) before use
  int rc = dt_compress_begin(master, snap, ef, cseg, cstart, cend, nchunks, nseg, seg_len, ws, 1, st);
  if (rc) return rc;
  // below 2^31 elements there is one index window, so the kept indices are plain flat indices
  rc = dt_compress_finish(ef, cseg, cstart, cend, nchunks, nseg, ws, k_fraction, adaptive, out_idx, out_val, out_q,
                          out_scales, quant_block, capacity, nullptr, 1, nullptr, st);
  if (rc) return rc;
  if (stats_out) return dt_compress_export_stats(ws, nseg, nchunks, stats_out, st);
  return 0;
}
