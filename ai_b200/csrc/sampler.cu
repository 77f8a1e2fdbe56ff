// Logits-in token sampler (sm_100a), one CTA per row.
//
// Reference semantics: GGUFEngine._pick (`ramvi/engine/ramvi_engine/core/gengine.py:452-469`) with the
// bitmask of Constraint.apply (`generation/constrain.py:146-148`): greedy = first index among the maxima;
// sampling = softmax(l.double()/T) -> descending order -> keep while the exclusive cumsum < top_p ->
// renormalise -> numpy Generator.choice with a uniform u (index = #(cdf <= u)).
// Extensions without a reference counterpart (the reference rejects them, server/validation.py:78-85):
// repetition penalty (l<0 ? l*r : l/r over the set of prior ids), presence/frequency penalties
// (l -= f*count + p*[count>0]) applied first, and top-k (keep z >= k-th largest) before top-p.
//
// Algorithm per row (no full sort of the vocabulary):
//  1. penalties via a sorted prior-id table + a vocabulary bitmap in shared memory (O(1) test per token);
//  2. greedy: block argmax;
//  3. top-k threshold by 4-pass radix select on order-preserving 32-bit keys of the logits;
//  4. candidates = the top min(k, CMAX) keys (same radix select); histograms use warp-aggregated shared
//     atomics (__match_any_sync), since logit keys crowd into a few buckets;
//  5. the candidates are gathered, bitonic-sorted by (key desc, index asc), and the nucleus cut,
//     renormalisation and inverse CDF are evaluated in float64 with a fixed-order block scan against the
//     softmax denominator from a fixed-order reduction -- deterministic run to run. If the nucleus (or, at
//     top_p = 1, the sampled point) lies beyond the CMAX largest logits the row sets AIB_DEV_SAMPLER_CAP.
#include <algorithm>
#include <climits>
#include "common.cuh"

namespace aib {
namespace samp {

constexpr int kThreads = 1024;
constexpr int CMAX = 8192;
constexpr int PMAX = 4096;

AIB_DEV uint32_t fkey(float f) {
  if (f != f) return 0u;  // NaN sorts last
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
AIB_DEV float key_value(uint32_t k) { return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k); }

struct Row {
  const float* l;
  const uint32_t* mask;  // may be null
  const uint32_t* bitmap;
  const int* pid;  // sorted prior ids (valid only), n_pid entries
  int n_pid;
  float rep, pres, freq;
};

// penalised + masked logit of token v whose raw logit is x
AIB_DEV float adjust(const Row& r, int v, float x) {
  if (r.mask && !((r.mask[v >> 5] >> (v & 31)) & 1u)) return -INFINITY;
  if ((r.bitmap[v >> 5] >> (v & 31)) & 1u) {
    int lo = 0, hi = r.n_pid;  // count = occurrences of v in the sorted prior list
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (r.pid[mid] < v) lo = mid + 1; else hi = mid;
    }
    const int a = lo;
    hi = r.n_pid;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (r.pid[mid] <= v) lo = mid + 1; else hi = mid;
    }
    const int cnt = lo - a;
    if (r.rep != 1.0f) x = (x < 0.0f) ? __fmul_rn(x, r.rep) : __fdiv_rn(x, r.rep);
    if (r.pres != 0.0f || r.freq != 0.0f)
      x = __fsub_rn(x, __fadd_rn(__fmul_rn(static_cast<float>(cnt), r.freq), r.pres));
  }
  return x;
}

// Eight consecutive raw logits from v0 (two 16-byte loads when the row is 16-byte aligned).
AIB_DEV void load8(const Row& r, int V, int v0, float* x) {
  if ((reinterpret_cast<uintptr_t>(r.l) & 15) == 0 && v0 + 8 <= V) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(r.l + v0));
    const float4 b = __ldg(reinterpret_cast<const float4*>(r.l + v0 + 4));
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = (v0 + i < V) ? __ldg(r.l + v0 + i) : 0.0f;
  }
}

// Visit every token of the row: f(v, adjusted logit). Each thread reads 8 consecutive logits per round,
// so a pass keeps ~8K loads in flight in the block.
template <typename F>
AIB_DEV void for_each_value(const Row& r, int V, F&& f) {
  for (int base = 0; base < V; base += kThreads * 8) {
    const int v0 = base + threadIdx.x * 8;
    float x[8];
    load8(r, V, v0, x);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (v0 + i < V) f(v0 + i, adjust(r, v0 + i, x[i]));
  }
}

template <typename T>
AIB_DEV T block_sum_fixed(T v, T* red) {  // deterministic: fixed lanes, fixed warp order
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T s = 0;
  for (int i = 0; i < kThreads / 32; ++i) s += red[i];
  return s;
}

// Radix-select step on a 256-bucket histogram (buckets visited from 255 down): the digit d holding the
// `rem`-th largest key and the count of keys in higher buckets. Run by one full warp (lane l owns buckets
// 255-8l .. 248-8l); every lane returns the same result.
AIB_DEV void pick_bucket(const unsigned int* hist, int rem, int& digit, int& above) {
  const int lane = threadIdx.x & 31;
  int c[8], tot = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = static_cast<int>(hist[255 - 8 * lane - i]), tot += c[i];
  int incl = tot;  // inclusive prefix over lanes (descending bucket order)
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const int excl = incl - tot;
  // first lane whose inclusive count reaches rem
  const unsigned hit = __ballot_sync(0xffffffffu, incl >= rem);
  const int src = hit ? __ffs(hit) - 1 : 31;
  int d = 0, ab = 0;
  if (lane == src) {
    int cum = excl;
    int i = 0;
    for (; i < 7; ++i) {
      if (cum + c[i] >= rem) break;
      cum += c[i];
    }
    d = 255 - 8 * lane - i;
    ab = cum;
  }
  digit = __shfl_sync(0xffffffffu, d, src);
  above = __shfl_sync(0xffffffffu, ab, src);
}

struct __align__(16) Shared {
  double dred[32];
  float fred[32];
  int ired[32];
  unsigned int hist[256];
  int ncand;
  int ncand_total;  // size of the kept set (V, or the top-k set)
  uint32_t prefix;
};

// Key of the k-th largest value among tokens with key >= floor (ties at the boundary counted once each;
// every token whose key is >= the result is kept). 4 radix passes of 8 bits; warp-aggregated histogram.
AIB_DEV uint32_t select_kth(const Row& r, int V, int k, uint32_t floor, Shared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t prefix = 0u, pmask = 0u;
  int remaining = k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    __syncthreads();
    for (int i = tid; i < 256; i += kThreads) sh.hist[i] = 0u;
    __syncthreads();
    for (int base = 0; base < V; base += kThreads * 8) {  // uniform trip count: warp-wide match below
      const int v0 = base + tid * 8;
      float x[8];
      load8(r, V, v0, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int bucket = 256;  // "no bucket"
        if (v0 + i < V) {
          const uint32_t key = fkey(adjust(r, v0 + i, x[i]));
          if (key >= floor && (key & pmask) == prefix) bucket = static_cast<int>((key >> shift) & 0xFFu);
        }
        const unsigned peers = __match_any_sync(0xffffffffu, bucket);
        if (bucket != 256 && lane == __ffs(peers) - 1)
          atomicAdd(&sh.hist[bucket], static_cast<unsigned>(__popc(peers)));
      }
    }
    __syncthreads();
    if (tid < 32) {
      int d, cum;
      pick_bucket(sh.hist, remaining, d, cum);
      if (tid == 0) {
        sh.prefix = prefix | (static_cast<uint32_t>(d) << shift);
        sh.ired[0] = remaining - cum;
      }
    }
    __syncthreads();
    prefix = sh.prefix;
    remaining = sh.ired[0];
    pmask |= 0xFFu << shift;
  }
  __syncthreads();
  return prefix;
}

// The whole sampling of row b by one CTA of kThreads threads (dsm: smem_bytes(V) of dynamic shared memory).
AIB_DEV void sample_row_full(uint8_t* dsm, Shared& sh, const float* __restrict__ logits, int V, int ld,
                             const aib_sample_params& prm, const int32_t* __restrict__ prior, int n_prior,
                             const int32_t* __restrict__ bitmask, const double* __restrict__ us,
                             int64_t* __restrict__ out, int b) {
  const int words = (V + 31) >> 5;
  const int words_pad = (words + 3) & ~3;  // keeps every later array 16-byte aligned
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(dsm);
  int* pid = reinterpret_cast<int*>(bitmap + words_pad);
  uint32_t* ckey = reinterpret_cast<uint32_t*>(pid + PMAX);
  int* cidx = reinterpret_cast<int*>(ckey + CMAX);
  double* cp = reinterpret_cast<double*>(cidx + CMAX);
  const int tid = threadIdx.x;

  Row r;
  r.l = logits + static_cast<size_t>(b) * ld;
  r.mask = bitmask ? reinterpret_cast<const uint32_t*>(bitmask) + static_cast<size_t>(b) * words : nullptr;
  r.bitmap = bitmap;
  r.pid = pid;
  r.rep = prm.repetition_penalty;
  r.pres = prm.presence_penalty;
  r.freq = prm.frequency_penalty;
  // ---- 1. prior-id table (sorted) + bitmap
  for (int i = tid; i < words; i += kThreads) bitmap[i] = 0u;
  const bool penal = prior && n_prior > 0 &&
                     (prm.repetition_penalty != 1.0f || prm.presence_penalty != 0.0f || prm.frequency_penalty != 0.0f);
  int np2 = 1;
  while (np2 < n_prior) np2 <<= 1;
  if (!penal) np2 = 0;
  for (int i = tid; i < np2; i += kThreads) {
    int v = INT_MAX;
    if (i < n_prior) {
      const int x = prior[static_cast<size_t>(b) * n_prior + i];
      if (x >= 0 && x < V) v = x;
    }
    pid[i] = v;
  }
  __syncthreads();
  for (int k = 2; k <= np2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const int a = pid[i], c = pid[ixj];
          const bool up = (i & k) == 0;
          if ((a > c) == up) pid[i] = c, pid[ixj] = a;
        }
      }
      __syncthreads();
    }
  int nvalid = 0;
  for (int i = tid; i < np2; i += kThreads) nvalid += pid[i] != INT_MAX;
  nvalid = block_sum_fixed<int>(nvalid, sh.ired);
  r.n_pid = nvalid;
  for (int i = tid; i < nvalid; i += kThreads) atomicOr(&bitmap[pid[i] >> 5], 1u << (pid[i] & 31));
  __syncthreads();

  // ---- 2. max (and greedy argmax: first index among the maxima)
  float best = -INFINITY;
  int bi = INT_MAX;
  for_each_value(r, V, [&](int v, float x) {
    if (x > best || (x == best && v < bi)) best = x, bi = v;
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) best = ob, bi = oi;
  }
  if ((tid & 31) == 0) sh.fred[tid >> 5] = best, sh.ired[tid >> 5] = bi;
  __syncthreads();
  best = -INFINITY;
  bi = INT_MAX;
  for (int i = 0; i < kThreads / 32; ++i)
    if (sh.fred[i] > best || (sh.fred[i] == best && sh.ired[i] < bi)) best = sh.fred[i], bi = sh.ired[i];
  if (bi == INT_MAX) bi = 0;  // every logit NaN / masked: first token
  const float T = prm.temperature;
  if (!(T > 0.0f) || best == -INFINITY) {
    if (tid == 0) out[b] = bi;
    return;
  }
  const double Td = static_cast<double>(T);  // z = l.double() / T, as the reference
  const double Mz = static_cast<double>(best) / Td;

  // ---- 3. top-k threshold key (k-th largest, ties kept)
  const int topk = prm.top_k;
  const uint32_t thr_k = (topk > 0 && topk < V) ? select_kth(r, V, topk, 0u, sh) : 0u;

  // ---- softmax denominator over the kept set (fixed-order reduction)
  double part = 0.0;
  for_each_value(r, V, [&](int, float x) {
    if (fkey(x) >= thr_k && x != -INFINITY) part += exp(static_cast<double>(x) / Td - Mz);
  });
  const double Z = block_sum_fixed<double>(part, sh.dred);
  const double top_p = static_cast<double>(prm.top_p);

  // ---- 4. candidates: the CMAX largest keys of the kept set (all of them if it is smaller)
  uint32_t thr = thr_k;
  const int kept_max = (topk > 0 && topk < V) ? topk : V;
  if (kept_max > CMAX) thr = max(thr, select_kth(r, V, CMAX, thr_k, sh));

  // ---- 5. gather candidates (key >= thr, finite), sort, exact nucleus + inverse CDF
  __syncthreads();
  if (tid == 0) sh.ncand = 0, sh.ncand_total = kept_max;
  __syncthreads();
  for_each_value(r, V, [&](int v, float x) {
    const uint32_t k = fkey(x);
    if (k >= thr && x != -INFINITY) {
      const int slot = atomicAdd(&sh.ncand, 1);
      if (slot < CMAX) ckey[slot] = k, cidx[slot] = v;
    }
  });
  __syncthreads();
  int nc = min(sh.ncand, CMAX);  // ties at the CMAX-th key can add a few more; the extra ones are dropped
  int n2 = 1;
  while (n2 < nc) n2 <<= 1;
  for (int i = nc + tid; i < n2; i += kThreads) ckey[i] = 0u, cidx[i] = INT_MAX;
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1)  // bitonic sort: (key desc, idx asc)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n2; i += kThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint32_t ka = ckey[i], kb = ckey[ixj];
          const int ia = cidx[i], ib = cidx[ixj];
          const bool a_first = (ka > kb) || (ka == kb && ia < ib);
          const bool up = (i & k) == 0;
          if (a_first != up) ckey[i] = kb, ckey[ixj] = ka, cidx[i] = ib, cidx[ixj] = ia;
        }
      }
      __syncthreads();
    }
  for (int i = tid; i < nc; i += kThreads)  // probabilities in sorted order
    cp[i] = exp(static_cast<double>(key_value(ckey[i])) / Td - Mz) / Z;
  __syncthreads();
  // exclusive scan in a fixed order: contiguous segment per thread, then lanes, then warps
  const int per = (nc + kThreads - 1) / kThreads;
  const int a0 = min(nc, tid * per), a1 = min(nc, a0 + per);
  double seg = 0.0;
  for (int i = a0; i < a1; ++i) seg += cp[i];
  double incl = seg;
  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) sh.dred[warp] = incl;
  __syncthreads();
  double wbase = 0.0;
  for (int w = 0; w < warp; ++w) wbase += sh.dred[w];
  double run = wbase + incl - seg;
  for (int i = a0; i < a1; ++i) {
    const double pi = cp[i];
    cp[i] = run;  // exclusive prefix
    run += pi;
  }
  __syncthreads();
  int keep = 0;  // keep while exclusive cumsum < top_p
  for (int i = tid; i < nc; i += kThreads) keep += (top_p >= 1.0 || cp[i] < top_p) ? 1 : 0;
  keep = block_sum_fixed<int>(keep, sh.ired);
  keep = max(1, min(keep, nc));
  // the candidates must contain the nucleus: their total mass reaches top_p, or they are the whole kept set
  if (tid == 0 && nc < sh.ncand_total && (cp[nc - 1] + exp(static_cast<double>(key_value(ckey[nc - 1])) / Td - Mz) / Z) < min(top_p, 1.0 - 1e-12))
    set_status(AIB_DEV_SAMPLER_CAP);
  const double pl = exp(static_cast<double>(key_value(ckey[keep - 1])) / Td - Mz) / Z;
  const double S = cp[keep - 1] + pl;  // kept mass
  const double u = us ? us[b] : 0.5;
  int cntle = 0;  // index = #(cdf_i <= u), cdf_i = inclusive_i / S
  for (int i = tid; i < keep; i += kThreads) {
    const double incl_i = (i + 1 < keep) ? cp[i + 1] : S;
    cntle += (incl_i / S <= u) ? 1 : 0;
  }
  cntle = block_sum_fixed<int>(cntle, sh.ired);
  const int pick = min(cntle, keep - 1);
  if (tid == 0) out[b] = cidx[pick];
}

__global__ void __launch_bounds__(kThreads)
    sample_kernel(const float* __restrict__ logits, int V, int ld, aib_sample_params prm,
                  const int32_t* __restrict__ prior, int n_prior, const int32_t* __restrict__ bitmask,
                  const double* __restrict__ us, int64_t* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Shared sh;
  pdl_wait();
  sample_row_full(dsm, sh, logits, V, ld, prm, prior, n_prior, bitmask, us, out, blockIdx.x);
  pdl_trigger();
}

// ------------------------------------------------------------------------------ two-phase fast path
// Phase 1 (grid: slices x rows, kPartThreads threads): each CTA takes a slice of at most kSliceMax tokens of
// one row, applies mask and penalties (prior ids of the slice counted in shared memory), and writes
//   * its max logit and the first index holding it;
//   * zmax_s = max/T and zsum_s = sum exp(l/T - zmax_s) in float64 over the slice (the softmax
//     denominator when there is no top-k);
//   * its candidates: every token whose key is >= the slice's C-th largest key (at most kCandCap; a slice
//     with more ties than that flags overflow).
// Phase 2 (one CTA of kThreads per row) merges the slices in slice order (deterministic): greedy from the
// maxima; otherwise the N = top_k (or C) largest keys of the union are selected, sorted (key desc, index
// asc) and the nucleus and inverse CDF are evaluated as in sample_row_full. Whenever the result could
// depend on a token outside the union (top_k > C, an overflowing slice, or a nucleus that the N largest
// tokens do not cover) the row falls back to sample_row_full: same tokens in every case.
constexpr int kPartThreads = 256;
constexpr int kSliceMax = 1280;   // 5 tokens per thread
constexpr int kC = 64;            // candidates per slice (top_k <= kC uses the fast path)
constexpr int kCandCap = 128;     // candidate slots per slice (ties at the C-th key)
constexpr int kMaxSlices = 192;   // merge keeps ns * kCandCap keys in registers (24 per thread)

struct SlicePart {
  double zmax, zsum;
  float max;
  int arg, ncand, overflow;
};

static int n_slices(int V) { return (V + kSliceMax - 1) / kSliceMax > 148 ? (V + kSliceMax - 1) / kSliceMax : std::min(148, (V + 255) / 256); }

__global__ void __launch_bounds__(kPartThreads)
    sample_part_kernel(const float* __restrict__ logits, int V, int ld, aib_sample_params prm,
                       const int32_t* __restrict__ prior, int n_prior, const int32_t* __restrict__ bitmask,
                       SlicePart* __restrict__ parts, uint32_t* __restrict__ ckeys, int* __restrict__ cids) {
  __shared__ int cnt[kSliceMax];
  __shared__ unsigned int hist[256];
  __shared__ float fred[kPartThreads / 32];
  __shared__ int ired[kPartThreads / 32];
  __shared__ double dred[kPartThreads / 32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_rem, s_nc;
  const int sl = blockIdx.x, ns = gridDim.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (V + ns - 1) / ns;
  const int v0 = min(V, sl * per), v1 = min(V, v0 + per);
  const float* l = logits + static_cast<size_t>(b) * ld;
  const uint32_t* mask = bitmask ? reinterpret_cast<const uint32_t*>(bitmask) + static_cast<size_t>(b) * ((V + 31) >> 5) : nullptr;
  for (int i = tid; i < kSliceMax; i += kPartThreads) cnt[i] = 0;
  pdl_wait();
  __syncthreads();
  const bool penal = prior && n_prior > 0 &&
                     (prm.repetition_penalty != 1.0f || prm.presence_penalty != 0.0f || prm.frequency_penalty != 0.0f);
  if (penal)
    for (int i = tid; i < n_prior; i += kPartThreads) {
      const int x = prior[static_cast<size_t>(b) * n_prior + i];
      if (x >= v0 && x < v1) atomicAdd(&cnt[x - v0], 1);
    }
  __syncthreads();
  constexpr int E = kSliceMax / kPartThreads;
  float x[E];
  uint32_t key[E];
  float best = -INFINITY;
  int bi = INT_MAX;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int v = v0 + e * kPartThreads + tid;
    float xv = -INFINITY;
    if (v < v1) {
      xv = l[v];
      if (mask && !((mask[v >> 5] >> (v & 31)) & 1u)) {
        xv = -INFINITY;
      } else {
        const int c = cnt[v - v0];
        if (c > 0) {
          if (prm.repetition_penalty != 1.0f)
            xv = (xv < 0.0f) ? __fmul_rn(xv, prm.repetition_penalty) : __fdiv_rn(xv, prm.repetition_penalty);
          if (prm.presence_penalty != 0.0f || prm.frequency_penalty != 0.0f)
            xv = __fsub_rn(xv, __fadd_rn(__fmul_rn(static_cast<float>(c), prm.frequency_penalty), prm.presence_penalty));
        }
      }
      if (xv > best || (xv == best && v < bi)) best = xv, bi = v;
    }
    x[e] = xv;
    key[e] = v < v1 ? fkey(xv) : 0u;
  }
  // max / first argmax of the slice
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) best = ob, bi = oi;
  }
  if (lane == 0) fred[warp] = best, ired[warp] = bi;
  __syncthreads();
  best = -INFINITY;
  bi = INT_MAX;
  for (int w = 0; w < kPartThreads / 32; ++w)
    if (fred[w] > best || (fred[w] == best && ired[w] < bi)) best = fred[w], bi = ired[w];
  SlicePart* pp = parts + static_cast<size_t>(b) * ns + sl;
  const float T = prm.temperature;
  if (!(T > 0.0f)) {
    if (tid == 0) pp->max = best, pp->arg = bi, pp->ncand = 0, pp->overflow = 0, pp->zmax = 0.0, pp->zsum = 0.0;
    pdl_trigger();
    return;
  }
  // float64 partial softmax denominator over the slice (fixed-order reduction); only needed without top-k
  const bool has_k = prm.top_k > 0 && prm.top_k < V;
  const double Td = static_cast<double>(T);
  const double zm = best == -INFINITY ? 0.0 : static_cast<double>(best) / Td;
  double zs = 0.0;
  if (!has_k) {
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (x[e] != -INFINITY && e * kPartThreads + tid < v1 - v0) zs += exp(static_cast<double>(x[e]) / Td - zm);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zs += __shfl_xor_sync(0xffffffffu, zs, o);
    __syncthreads();
    if (lane == 0) dred[warp] = zs;
    __syncthreads();
    zs = 0.0;
    for (int w = 0; w < kPartThreads / 32; ++w) zs += dred[w];
  }
  // kc-th largest key of the slice (kc = top_k when it is at most kC, else kC): 4 radix passes over the
  // keys held in registers
  const int kc = min(has_k ? min(prm.top_k, kC) : kC, v1 - v0);
  uint32_t prefix = 0u, pmask = 0u;
  int rem = kc;
  for (int shift = 24; shift >= 0 && kc > 0; shift -= 8) {
    __syncthreads();
    hist[tid] = 0u;  // kPartThreads == 256 buckets
    __syncthreads();
#pragma unroll
    for (int e = 0; e < E; ++e) {
      int bucket = 256;
      if (e * kPartThreads + tid < v1 - v0 && (key[e] & pmask) == prefix) bucket = static_cast<int>((key[e] >> shift) & 0xFFu);
      const unsigned peers = __match_any_sync(0xffffffffu, bucket);
      if (bucket != 256 && lane == __ffs(peers) - 1) atomicAdd(&hist[bucket], static_cast<unsigned>(__popc(peers)));
    }
    __syncthreads();
    if (tid < 32) {
      int d, cum;
      pick_bucket(hist, rem, d, cum);
      if (tid == 0) {
        s_prefix = prefix | (static_cast<uint32_t>(d) << shift);
        s_rem = rem - cum;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    rem = s_rem;
    pmask |= 0xFFu << shift;
  }
  // candidates: keys >= the kc-th key (finite logits)
  if (tid == 0) s_nc = 0;
  __syncthreads();
  uint32_t* ck = ckeys + (static_cast<size_t>(b) * ns + sl) * kCandCap;
  int* ci = cids + (static_cast<size_t>(b) * ns + sl) * kCandCap;
  bool over = false;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int v = v0 + e * kPartThreads + tid;
    if (v < v1 && kc > 0 && key[e] >= prefix && x[e] != -INFINITY) {
      const int slot = atomicAdd(&s_nc, 1);
      if (slot < kCandCap) ck[slot] = key[e], ci[slot] = v; else over = true;
    }
  }
  over = __syncthreads_or(over);
  if (tid == 0) {
    pp->max = best;
    pp->arg = bi;
    pp->zmax = zm;
    pp->zsum = zs;
    pp->ncand = min(s_nc, kCandCap);
    pp->overflow = over ? 1 : 0;
  }
  pdl_trigger();
}

__global__ void __launch_bounds__(kThreads)
    sample_merge_kernel(const float* __restrict__ logits, int V, int ld, aib_sample_params prm,
                        const int32_t* __restrict__ prior, int n_prior, const int32_t* __restrict__ bitmask,
                        const double* __restrict__ us, int64_t* __restrict__ out, int ns,
                        const SlicePart* __restrict__ parts, const uint32_t* __restrict__ ckeys,
                        const int* __restrict__ cids) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ Shared sh;
  __shared__ SlicePart spart[kMaxSlices];
  __shared__ int soff[kMaxSlices + 1];  // exclusive prefix of the slices' candidate counts
  __shared__ float s_best;
  __shared__ int s_bi, s_over;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  for (int i = tid; i < ns; i += kThreads) spart[i] = parts[static_cast<size_t>(b) * ns + i];
  __syncthreads();
  // warp 0: global max / first argmax (slices in order), overflow flags, candidate offsets
  if (warp == 0) {
    float best = -INFINITY;
    int bi = INT_MAX, over = 0, run = 0;
    for (int i0 = 0; i0 < ns; i0 += 32) {
      const int i = i0 + lane;
      const bool ok = i < ns;
      const float m = ok ? spart[i].max : -INFINITY;
      const int a = ok ? spart[i].arg : INT_MAX;
      if (ok) over |= spart[i].overflow;
      if (m > best || (m == best && a < bi)) best = m, bi = a;
      int c = ok ? spart[i].ncand : 0, incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (ok) soff[i] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) best = ob, bi = oi;
    }
    over = __any_sync(0xffffffffu, over != 0);
    if (lane == 0) s_best = best, s_bi = bi, s_over = over, soff[ns] = run;
  }
  __syncthreads();
  const float best = s_best;
  int bi = s_bi;
  if (bi == INT_MAX) bi = 0;
  const float T = prm.temperature;
  if (!(T > 0.0f) || best == -INFINITY) {
    if (tid == 0) out[b] = bi;
    pdl_trigger();
    return;
  }
  const int topk = prm.top_k;
  const bool has_k = topk > 0 && topk < V;
  const int total = soff[ns];
  if (s_over || (has_k && topk > kC) || total > CMAX) {
    sample_row_full(dsm, sh, logits, V, ld, prm, prior, n_prior, bitmask, us, out, b);
    pdl_trigger();
    return;
  }
  const double Td = static_cast<double>(T), Mz = static_cast<double>(best) / Td;
  // compact the candidates into shared memory (warp per slice, lanes over the slice's list)
  // dynamic shared memory (smem_bytes(V) >= 128 KB): [0, 64K) all candidates (keys, ids), then reused for
  // the probabilities; [64K, 128K) the kept candidates (keys, ids)
  uint32_t* ak = reinterpret_cast<uint32_t*>(dsm);
  int* ai = reinterpret_cast<int*>(ak + CMAX);
  uint32_t* ckey = reinterpret_cast<uint32_t*>(ai + CMAX);
  int* cidx = reinterpret_cast<int*>(ckey + CMAX);
  double* cp = reinterpret_cast<double*>(dsm);  // written only after the gather has consumed ak / ai
  for (int sl = warp; sl < ns; sl += kThreads / 32) {
    const int n = spart[sl].ncand, o = soff[sl];
    const size_t src = (static_cast<size_t>(b) * ns + sl) * kCandCap;
    for (int j = lane; j < n; j += 32) {
      ak[o + j] = __ldcg(ckeys + src + j);
      ai[o + j] = __ldcg(cids + src + j);
    }
  }
  __syncthreads();
  // N-th largest key of the union (radix select over the compact list)
  const int N = has_k ? topk : kC;
  uint32_t prefix = 0u, pmask = 0u;
  int rem = min(N, total);
  const int rounds = (total + kThreads - 1) / kThreads;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kThreads) sh.hist[i] = 0u;
    __syncthreads();
    for (int r2 = 0; r2 < rounds; ++r2) {
      const int i = r2 * kThreads + tid;
      int bucket = 256;
      if (i < total && (ak[i] & pmask) == prefix) bucket = static_cast<int>((ak[i] >> shift) & 0xFFu);
      const unsigned peers = __match_any_sync(0xffffffffu, bucket);
      if (bucket != 256 && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[bucket], static_cast<unsigned>(__popc(peers)));
    }
    __syncthreads();
    if (tid < 32) {
      int d, cum;
      pick_bucket(sh.hist, rem, d, cum);
      if (tid == 0) {
        sh.prefix = prefix | (static_cast<uint32_t>(d) << shift);
        sh.ired[0] = rem - cum;
      }
    }
    __syncthreads();
    prefix = sh.prefix;
    rem = sh.ired[0];
    pmask |= 0xFFu << shift;
  }
  const uint32_t thr = prefix;
  if (tid == 0) sh.ncand = 0;
  __syncthreads();
  for (int i = tid; i < total; i += kThreads)
    if (ak[i] >= thr) {
      const int slot = atomicAdd(&sh.ncand, 1);
      ckey[slot] = ak[i], cidx[slot] = ai[i];
    }
  __syncthreads();
  const int nc = sh.ncand;
  if (nc > 256) {  // many ties at the boundary key: the parallel single-CTA algorithm handles them
    sample_row_full(dsm, sh, logits, V, ld, prm, prior, n_prior, bitmask, us, out, b);
    pdl_trigger();
    return;
  }
  // sort (key desc, index asc): one warp when it fits, else a block bitonic sort
  if (nc <= 32) {
    if (warp == 0) {
      uint32_t k = lane < nc ? ckey[lane] : 0u;
      int id = lane < nc ? cidx[lane] : INT_MAX;
#pragma unroll
      for (int kk = 2; kk <= 32; kk <<= 1)
#pragma unroll
        for (int j = kk >> 1; j > 0; j >>= 1) {
          const uint32_t ok = __shfl_xor_sync(0xffffffffu, k, j);
          const int oi = __shfl_xor_sync(0xffffffffu, id, j);
          const bool lower = (lane & j) == 0;        // this lane holds the first of the pair
          const bool up = (lane & kk) == 0;          // ascending block of the bitonic network ("first" = larger)
          const bool mine_first = (k > ok) || (k == ok && id < oi);
          const bool keep_mine = (lower == up) ? mine_first : !mine_first;
          if (!keep_mine) k = ok, id = oi;
        }
      if (lane < nc) ckey[lane] = k, cidx[lane] = id;
    }
    __syncthreads();
  } else {
    int n2 = 1;
    while (n2 < nc) n2 <<= 1;
    for (int i = nc + tid; i < n2; i += kThreads) ckey[i] = 0u, cidx[i] = INT_MAX;
    __syncthreads();
    for (int k = 2; k <= n2; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < n2; i += kThreads) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const uint32_t ka = ckey[i], kb = ckey[ixj];
            const int ia = cidx[i], ib = cidx[ixj];
            const bool a_first = (ka > kb) || (ka == kb && ia < ib);
            const bool up = (i & k) == 0;
            if (a_first != up) ckey[i] = kb, ckey[ixj] = ka, cidx[i] = ib, cidx[ixj] = ia;
          }
        }
        __syncthreads();
      }
  }
  // softmax denominator: over the kept top-k set (sorted order), or over the whole row from the slices.
  // The exponentials are evaluated in parallel (ep: candidates in sorted order, zt: slice terms); one thread
  // then adds them in a fixed order.
  double* ep = cp + 256;  // nc <= 256
  double* zt = cp + 512;  // ns <= kMaxSlices
  for (int i = tid; i < nc; i += kThreads) ep[i] = exp(static_cast<double>(key_value(ckey[i])) / Td - Mz);
  if (!has_k)
    for (int s2 = tid; s2 < ns; s2 += kThreads)
      zt[s2] = spart[s2].max != -INFINITY ? spart[s2].zsum * exp(spart[s2].zmax - Mz) : 0.0;
  __syncthreads();
  if (tid == 0) {
    double Z = 0.0;
    if (has_k) {
      for (int i = 0; i < nc; ++i) Z += ep[i];
    } else {
      for (int s2 = 0; s2 < ns; ++s2)
        if (spart[s2].max != -INFINITY) Z += zt[s2];
    }
    // probabilities and their exclusive prefix sums in sorted order (fixed order)
    double run = 0.0;
    for (int i = 0; i < nc; ++i) {
      const double pi = ep[i] / Z;
      cp[i] = run;
      run += pi;
    }
    sh.dred[0] = run;  // mass of all candidates
    sh.dred[1] = Z;
  }
  __syncthreads();
  const double top_p = static_cast<double>(prm.top_p), cand_mass = sh.dred[0], Z = sh.dred[1];
  // without top-k the candidates are the N largest logits of the row: fall back when the nucleus may extend
  // past them (their mass does not reach top_p and the row has more tokens)
  if (!has_k && nc < V && cand_mass < min(top_p, 1.0 - 1e-12)) {
    __syncthreads();
    sample_row_full(dsm, sh, logits, V, ld, prm, prior, n_prior, bitmask, us, out, b);
    pdl_trigger();
    return;
  }
  if (tid == 0) {
    int keep = 0;  // keep while exclusive cumsum < top_p
    for (int i = 0; i < nc; ++i) keep += (top_p >= 1.0 || cp[i] < top_p) ? 1 : 0;
    keep = max(1, min(keep, nc));
    const double pl = ep[keep - 1] / Z;
    const double S = cp[keep - 1] + pl;
    const double u = us ? us[b] : 0.5;
    int cntle = 0;  // index = #(cdf_i <= u)
    for (int i = 0; i < keep; ++i) {
      const double incl_i = (i + 1 < keep) ? cp[i + 1] : S;
      cntle += (incl_i / S <= u) ? 1 : 0;
    }
    out[b] = cidx[min(cntle, keep - 1)];
  }
  pdl_trigger();
}

static size_t smem_bytes(int V) {
  const size_t words = ((static_cast<size_t>(V) + 31) / 32 + 3) & ~static_cast<size_t>(3);
  return words * 4 + PMAX * 4 + CMAX * 4 + CMAX * 4 + CMAX * 8;
}

}  // namespace samp
}  // namespace aib

using namespace aib;

extern "C" {

size_t aib_sample_workspace(int B, int V) {
  if (B <= 0 || V <= 0) return 0;
  const size_t ns = static_cast<size_t>(samp::n_slices(V));
  return static_cast<size_t>(B) * ns * (sizeof(samp::SlicePart) + samp::kCandCap * 8) + 256;
}

int aib_sample(const float* logits, int B, int V, int ld, const aib_sample_params* params, const int32_t* prior,
               int n_prior, const int32_t* bitmask, const double* u, int64_t* out_ids, void* ws, size_t ws_bytes,
               void* stream) {
  if (!logits || !params || !out_ids || B <= 0 || V <= 0 || ld < V)
    return fail(AIB_EINVAL, "aib_sample: bad arguments (B=%d V=%d ld=%d)", B, V, ld);
  if (n_prior < 0 || n_prior > samp::PMAX) return fail(AIB_EINVAL, "aib_sample: n_prior must be in 0..%d", samp::PMAX);
  const aib_sample_params& p = *params;
  if (p.temperature > 0.0f && !u) return fail(AIB_EINVAL, "aib_sample: sampling needs the uniform draws u");
  if (p.temperature > 0.0f && !(p.top_p > 0.0f)) return fail(AIB_EINVAL, "aib_sample: top_p must be > 0");
  if (!(p.repetition_penalty > 0.0f)) return fail(AIB_EINVAL, "aib_sample: repetition_penalty must be > 0");
  const size_t smem = samp::smem_bytes(V);
  if (smem > 227 * 1024) return fail(AIB_ENOTSUP, "aib_sample: vocabulary of %d too large", V);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ws && ws_bytes >= aib_sample_workspace(B, V) && B <= 65535 && samp::n_slices(V) <= samp::kMaxSlices) {
    if (reinterpret_cast<uintptr_t>(ws) & 15) return fail(AIB_EINVAL, "aib_sample: workspace must be 16-byte aligned");
    const int ns = samp::n_slices(V);
    samp::SlicePart* parts = static_cast<samp::SlicePart*>(ws);
    uint32_t* ck = reinterpret_cast<uint32_t*>(parts + static_cast<size_t>(B) * ns);
    int* ci = reinterpret_cast<int*>(ck + static_cast<size_t>(B) * ns * samp::kCandCap);
    int rc = launch(samp::sample_part_kernel, dim3(ns, B), dim3(samp::kPartThreads), 0, s, "aib_sample (slices)",
                    logits, V, ld, p, prior, n_prior, bitmask, parts, ck, ci);
    if (rc) return rc;
    rc = allow_smem(samp::sample_merge_kernel, smem);
    if (rc) return rc;
    return launch(samp::sample_merge_kernel, dim3(B), dim3(samp::kThreads), smem, s, "aib_sample (merge)", logits, V,
                  ld, p, prior, n_prior, bitmask, u, out_ids, ns, static_cast<const samp::SlicePart*>(parts),
                  static_cast<const uint32_t*>(ck), static_cast<const int*>(ci));
  }
  const int rc = allow_smem(samp::sample_kernel, smem);
  if (rc) return rc;
  return launch(samp::sample_kernel, dim3(B), dim3(samp::kThreads), smem, s, "aib_sample", logits, V, ld, p, prior,
                n_prior, bitmask, u, out_ids);
}

}  // extern "C"
