// B200-native token sampler (sm_100a).
//
// One launch samples every row of a batch.  Each row is handled by a thread
// block cluster of C CTAs; CTA r streams columns [r*per_cta, (r+1)*per_cta)
// of the row once from HBM through a 4-stage bulk-copy (TMA) pipeline into
// shared memory, and the cluster leader merges the CTAs' results through
// distributed shared memory.  Per row, by mode:
//
//   GREEDY (temperature == 0; reference sampler.py:60-70)
//       first-index argmax of the penalised logits (NaN counts as max).
//   FAST   (0 < top_k <= kFastK; reference sampler.py:73-89, 110-133)
//       single-pass threshold filter: every CTA keeps, in a shared-memory
//       candidate buffer, all logits >= a running lower bound of its local
//       k-th largest value; the bound is raised by an in-shared-memory radix
//       select whenever the buffer would overflow (the vocabulary is never
//       sorted).  The leader selects the global k-th value over the union,
//       then runs top-p and the inverse-CDF draw on the few survivors.
//   GENERAL (top-k disabled or larger than kFastK): reported as
//       NS_ERR_UNSUPPORTED by this version.
//
// Penalties (reference sampler.py:93-108 plus presence/frequency): before the
// stream starts, each CTA hashes the row's history ids that fall in its column
// range (id -> count) and buckets the distinct ids by tile.  When a tile
// lands in shared memory the bucket's logits are penalised in fp32 (IEEE
// division / multiplication / subtraction, never contracted into FMAs), kept
// aside, and their slots overwritten with -inf so the streaming pass sees
// only un-penalised columns.
//
// Temperature is applied without a per-element division: y = x / T is
// monotone in x, so the k-th largest y is rn(x_k / T) and the survivors
// {rn(x / T) >= rn(x_k / T)} are exactly {x >= x_lo} for the smallest x_lo
// with rn(x_lo / T) >= rn(x_k / T), found by a short search over float keys.
// Negative temperatures are handled by negating x (rn(-x / -T) = rn(x / T)).
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "ns_common.cuh"
#include "ns_sampler.h"

namespace cg = cooperative_groups;

namespace ns {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 4;
constexpr int kTileBytes = 16384;
constexpr int kStageStride = kTileBytes + 128;
constexpr int kCap = 1024;       // per-CTA candidate buffer (entries)
constexpr int kFastK = 512;      // largest top_k served by the single-pass path
constexpr int kBins = 256;       // radix digit = 8 bits
constexpr int kHashMax = 4096;   // distinct history ids per CTA (power of two)
constexpr int kMaxCluster = 8;
constexpr unsigned kFull = 0xFFFFFFFFu;

enum : int { MODE_GREEDY = 0, MODE_FAST = 1, MODE_GENERAL = 2 };
enum : int { F_NAN = 1, F_BADID = 2, F_HIST = 4, F_OVF = 8, F_TIMEOUT = 16, F_UNSUP = 32 };

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <int DT>
struct Elem;
template <>
struct Elem<NS_DTYPE_F32> {
  using raw = uint32_t;
  static constexpr int size = 4;
  static constexpr raw ninf = 0xFF800000u, pinf = 0x7F800000u;
  static __device__ __forceinline__ float widen(raw b) { return __uint_as_float(b); }
};
template <>
struct Elem<NS_DTYPE_BF16> {
  using raw = uint16_t;
  static constexpr int size = 2;
  static constexpr raw ninf = 0xFF80u, pinf = 0x7F80u;
  static __device__ __forceinline__ float widen(raw b) { return __uint_as_float(uint32_t(b) << 16); }
};
template <>
struct Elem<NS_DTYPE_F16> {
  using raw = uint16_t;
  static constexpr int size = 2;
  static constexpr raw ninf = 0xFC00u, pinf = 0x7C00u;
  static __device__ __forceinline__ float widen(raw b) { return __half2float(__ushort_as_half(b)); }
};

// ---------------------------------------------------------------------------
// shared-memory state
// ---------------------------------------------------------------------------
struct Misc {
  int n_cand;      // entries in the candidate buffer
  int pad2;
  int flags;       // F_* bits
  int n_unique;    // distinct history ids in this CTA's range
  float tau;       // filter threshold (negated domain when T < 0)
  int r_digit;     // radix-select broadcast
  int r_krem;
  int r_total;
  int n_merge;     // leader: survivors gathered from the cluster
  int choose;      // leader: inverse-CDF pick
  float g_best;    // greedy result of this CTA
  int g_idx;       // ... as a column of this call's logits
  int pad0, pad1;
  double d_red[kWarps];
  float f_red[kWarps];
  int i_red[kWarps];
  int roff[kMaxCluster * 2 + 2];
  int rc0[kMaxCluster * 2 + 2];
};

struct KArgs {
  const void* logits;
  int64_t vocab;         // columns read per row
  int64_t row_stride;    // elements between rows
  int64_t vocab_offset;  // global id of column 0 (vocab-parallel slices)
  int64_t vocab_total;   // global vocabulary size
  const int32_t* hist_ids;
  const int64_t* hist_offsets;
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* rep;
  const float* pres;
  const float* freq;
  const float* uniforms;
  uint64_t seed;
  uint64_t offset;
  int64_t* out_ids;
  int per_cta;     // columns per CTA, a multiple of the 16-byte vector width
  int tiles_max;   // tiles per CTA (upper bound)
  int hash_slots;  // power of two
  int uniq_cap;    // distinct ids the bucket arrays hold
  int merge_cap;   // leader merge area (entries)
  int64_t max_history;  // host bound on any row's history length
  uint32_t off_bar, off_cx, off_cid, off_hist, off_hkey, off_hcnt, off_bcol, off_bcnt, off_bx, off_toff,
      off_tfill, off_misc;
};

template <int DT>
struct Ctx {
  using E = Elem<DT>;
  static constexpr int ES = E::size;
  static constexpr int VE = 16 / ES;         // elements per 16-byte vector
  static constexpr int TE = kTileBytes / ES;  // elements per tile

  uint8_t* stages;
  uint64_t* bar;
  float* cx;
  int* cid;
  uint32_t* hist;
  int* hkey;
  int* hcnt;
  int* bcol;
  int* bcnt;
  float* bx;
  int* toff;
  int* tfill;
  Misc* m;

  const uint8_t* rowp;  // column 0 of this row
  int c0, c1;           // this CTA's columns
  int n_tiles;
  int K;
  bool neg;
  float Tabs;

  __device__ __forceinline__ int tile_len(int t) const { return min(TE, c1 - (c0 + t * TE)); }
  // Elements before the first 16-byte aligned column of the tile, and the
  // shared-memory slot of the tile's first column (so the aligned body lands
  // on a 16-byte boundary).
  __device__ __forceinline__ int tile_head(int t) const {
    const uintptr_t a = reinterpret_cast<uintptr_t>(rowp) + uintptr_t(c0 + t * TE) * ES;
    return min(int(((16u - (a & 15u)) & 15u) / ES), tile_len(t));
  }
  __device__ __forceinline__ int tile_lead(int t) const { return (VE - tile_head(t)) % VE; }
  __device__ __forceinline__ uint8_t* stage(int t) const { return stages + (t % kStages) * kStageStride; }
};

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  return a > b || (a == b && ia < ib);
}

// repetition (reference sampler.py:104-107), then frequency and presence; each
// a separately rounded fp32 operation.
__device__ __forceinline__ float penalize(float x, int count, float rep, float pres, float freq) {
  if (rep != 1.0f) x = (x < 0.0f) ? __fmul_rn(x, rep) : __fdiv_rn(x, rep);
  if (freq != 0.0f) x = __fsub_rn(x, __fmul_rn(freq, (float)count));
  if (pres != 0.0f) x = __fsub_rn(x, pres);
  return x;
}

template <int DT>
__device__ __forceinline__ void unpack16(const uint4& v, float (&x)[Ctx<DT>::VE]) {
  using E = Elem<DT>;
  if constexpr (DT == NS_DTYPE_F32) {
    x[0] = __uint_as_float(v.x);
    x[1] = __uint_as_float(v.y);
    x[2] = __uint_as_float(v.z);
    x[3] = __uint_as_float(v.w);
  } else {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = E::widen(uint16_t(w[i] & 0xFFFFu));
      x[2 * i + 1] = E::widen(uint16_t(w[i] >> 16));
    }
  }
}

// Reserve n buffer slots without ever exceeding kCap; -1 if they do not fit.
__device__ __forceinline__ int reserve_slots(Misc* m, int n) {
  int old = *reinterpret_cast<volatile int*>(&m->n_cand);
  while (true) {
    if (old + n > kCap) return -1;
    const int prev = atomicCAS(&m->n_cand, old, old + n);
    if (prev == old) return old;
    old = prev;
  }
}

// Warp-aggregated append; all 32 lanes must call it.  Returns true (in every
// lane) if the warp's entries did not fit; nothing is written then.
template <int DT>
__device__ __forceinline__ bool warp_append(const Ctx<DT>& c, bool want, float x, int col) {
  const unsigned mask = __ballot_sync(kFull, want);
  if (!mask) return false;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(mask) - 1;
  int base = 0;
  if (lane == leader) base = reserve_slots(c.m, __popc(mask));
  base = __shfl_sync(kFull, base, leader);
  if (base >= 0 && want) {
    const int pos = base + __popc(mask & lanemask_lt());
    c.cx[pos] = x;
    c.cid[pos] = col;
  }
  return base < 0;
}

// K-th largest (1-based) of the values visited by `for_each` (called by every
// thread of the CTA with a per-thread share).  Returns false if fewer than K
// values were visited.  8-bit MSB-first radix select in shared memory.
template <int DT, class ForEach>
__device__ bool radix_kth(const Ctx<DT>& c, int K, ForEach for_each, uint32_t* out_key) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  int krem = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < kBins; i += kThreads) c.hist[i] = 0;
    __syncthreads();
    for_each([&](float x) {
      const uint32_t k = f2key(x);
      if ((k & pmask) == prefix) atomicAdd(&c.hist[(k >> shift) & 0xFFu], 1u);
    });
    __syncthreads();
    if (warp == 0) {
      uint32_t cnt[8];
      uint32_t local = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cnt[q] = c.hist[255 - 8 * lane - q];
        local += cnt[q];
      }
      uint32_t incl = local;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
      }
      const uint32_t excl = incl - local;
      const unsigned b = __ballot_sync(kFull, incl >= uint32_t(krem));
      if (b == 0) {
        if (lane == 31) {
          c.m->r_digit = -1;
          c.m->r_total = int(incl);
        }
      } else if (lane == __ffs(b) - 1) {
        uint32_t cum = excl;
        int d = 255 - 8 * lane, kr = krem;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (cum + cnt[q] >= uint32_t(krem)) {
            d = 255 - 8 * lane - q;
            kr = krem - int(cum);
            break;
          }
          cum += cnt[q];
        }
        c.m->r_digit = d;
        c.m->r_krem = kr;
      }
    }
    __syncthreads();
    const int d = c.m->r_digit;
    if (d < 0) return false;
    prefix |= uint32_t(d) << shift;
    pmask |= 0xFFu << shift;
    krem = c.m->r_krem;
    __syncthreads();
  }
  *out_key = prefix;
  return true;
}

// Smallest x with rn(x / T) >= rn(xk / T) (T > 0): the filter bound that keeps
// every value whose scaled logit ties the k-th.  Gallop then bisect on keys.
__device__ float scaled_lower_bound(float xk, float T) {
  if (!(xk > -INFINITY)) return -INFINITY;
  const float ty = __fdiv_rn(xk, T);
  if (!(ty > -INFINITY)) return -INFINITY;
  const uint32_t kmin = f2key(-INFINITY);
  uint32_t hi = f2key(xk), lo = kmin;
  uint32_t step = 1;
  while (true) {
    const uint32_t cand = (hi - kmin > step) ? hi - step : kmin;
    if (__fdiv_rn(key2f(cand), T) >= ty) {
      hi = cand;
      if (cand == kmin) return -INFINITY;
      step <<= 1;
      if (step == 0) step = 0x80000000u;
    } else {
      lo = cand;
      break;
    }
  }
  while (hi - lo > 1) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (__fdiv_rn(key2f(mid), T) >= ty)
      hi = mid;
    else
      lo = mid;
  }
  return key2f(hi);
}

// Keep the buffer entries for which keep(x, col) holds (in place).
template <int DT, class Keep>
__device__ void compact_buffer(const Ctx<DT>& c, Keep keep) {
  constexpr int PER = kCap / kThreads;
  const int tid = threadIdx.x;
  const int n = c.m->n_cand;
  float xs[PER];
  int cs[PER];
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int i = q * kThreads + tid;
    xs[q] = (i < n) ? c.cx[i] : -INFINITY;
    cs[q] = (i < n) ? c.cid[i] : 0;
  }
  __syncthreads();
  if (tid == 0) c.m->n_cand = 0;
  __syncthreads();
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int i = q * kThreads + tid;
    warp_append(c, (i < n) && keep(xs[q], cs[q]), xs[q], cs[q]);
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// producer: one bulk copy per tile (plain loads for an unaligned head / tail)
// ---------------------------------------------------------------------------
template <int DT>
__device__ void issue_tile(const Ctx<DT>& c, int t, uint64_t policy) {
  using E = Elem<DT>;
  constexpr int ES = E::size;
  const int s = t % kStages;
  uint8_t* dst = c.stage(t);
  const int len = c.tile_len(t);
  const int head = c.tile_head(t);
  const int body = (((len - head) * ES) & ~15) / ES;
  const int tail = len - head - body;
  const int lead = c.tile_lead(t);
  const typename E::raw* src = reinterpret_cast<const typename E::raw*>(c.rowp) + (c.c0 + t * Ctx<DT>::TE);
  typename E::raw* d = reinterpret_cast<typename E::raw*>(dst);
  for (int q = 0; q < head; ++q) d[lead + q] = src[q];
  for (int q = 0; q < tail; ++q) d[lead + head + body + q] = src[head + body + q];
  const uint32_t bytes = uint32_t(body) * ES;
  mbar_arrive_expect_tx(&c.bar[s], bytes);
  if (bytes) bulk_g2s(d + lead + head, src + head, bytes, &c.bar[s], policy);
}

// ---------------------------------------------------------------------------
// consumers
// ---------------------------------------------------------------------------
// FAST: append every valid value >= tau (tile slots, then the tile's penalised
// history entries).  NaN or +inf in a sampled row flags F_NAN.  Returns true
// if any of this thread's warp appends did not fit.
template <int DT>
__device__ bool fast_tile(const Ctx<DT>& c, int t, float tau) {
  bool ovf = false;
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  const uint8_t* st = c.stage(t);
  const int len = c.tile_len(t), lead = c.tile_lead(t);
  const int n_groups = (lead + len + VE - 1) / VE;
  const int iters = (n_groups + kThreads - 1) / kThreads;
  const int colbase = t * TE - lead;
  for (int it = 0; it < iters; ++it) {
    const int q = it * kThreads + threadIdx.x;
    float x[VE];
    bool hot = false;
    if (q < n_groups) {
      const uint4 v = *reinterpret_cast<const uint4*>(st + q * 16);
      unpack16<DT>(v, x);
#pragma unroll
      for (int i = 0; i < VE; ++i) {
        if (c.neg) x[i] = -x[i];
        hot |= !(x[i] < tau);
      }
    } else {
#pragma unroll
      for (int i = 0; i < VE; ++i) x[i] = -INFINITY;
    }
    if (__any_sync(kFull, hot)) {
#pragma unroll
      for (int i = 0; i < VE; ++i) {
        const int e = q * VE + i;
        const bool valid = (q < n_groups) && e >= lead && e < lead + len;
        const float xi = x[i];
        const bool bad = valid && (xi != xi || xi == INFINITY);
        if (bad) atomicOr(&c.m->flags, F_NAN);
        ovf |= warp_append(c, valid && !bad && xi >= tau && xi > -INFINITY, xi, colbase + e);
      }
    }
  }
  const int b0 = c.toff[t], b1 = c.toff[t + 1];
  const int biters = (b1 - b0 + kThreads - 1) / kThreads;
  for (int it = 0; it < biters; ++it) {
    const int j = b0 + it * kThreads + threadIdx.x;
    const bool in = j < b1;
    const float xi = in ? c.bx[j] : -INFINITY;
    const int col = in ? c.bcol[j] : 0;
    const bool bad = in && (xi != xi || xi == INFINITY);
    if (bad) atomicOr(&c.m->flags, F_NAN);
    ovf |= warp_append(c, in && !bad && xi >= tau && xi > -INFINITY, xi, col);
  }
  return ovf;
}

// Values of tile t that the filter would consider at threshold tau.
template <int DT, class F>
__device__ __forceinline__ void visit_tile(const Ctx<DT>& c, int t, float tau, F f) {
  constexpr int VE = Ctx<DT>::VE;
  const uint8_t* st = c.stage(t);
  const int len = c.tile_len(t), lead = c.tile_lead(t);
  const int n_groups = (lead + len + VE - 1) / VE;
  for (int q = threadIdx.x; q < n_groups; q += kThreads) {
    float x[VE];
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int e = q * VE + i;
      const float xi = c.neg ? -x[i] : x[i];
      if (e >= lead && e < lead + len && xi >= tau && xi > -INFINITY && xi != INFINITY) f(xi);
    }
  }
  for (int j = c.toff[t] + threadIdx.x; j < c.toff[t + 1]; j += kThreads) {
    const float xi = c.bx[j];
    if (xi >= tau && xi > -INFINITY && xi != INFINITY) f(xi);
  }
}

// Re-process tile t after its appends overflowed the buffer (or directly,
// while no threshold exists yet): drop the tile's entries, select the K-th
// largest over buffer + tile, raise tau, compact, append again.
template <int DT>
__device__ void select_tile(const Ctx<DT>& c, int t) {
  constexpr int TE = Ctx<DT>::TE;
  const int tid = threadIdx.x;
  const float tau_old = c.m->tau;
  const int lo = t * TE, hi = lo + c.tile_len(t);
  const int n_buf = c.m->n_cand;
  auto for_each = [&](auto f) {
    for (int i = tid; i < n_buf; i += kThreads) {
      const int col = c.cid[i];
      if (col < lo || col >= hi) f(c.cx[i]);
    }
    visit_tile(c, t, tau_old, f);
  };
  uint32_t key = 0;
  const bool have = radix_kth(c, c.K, for_each, &key);
  if (tid == 0) c.m->tau = have ? fmaxf(tau_old, scaled_lower_bound(key2f(key), c.Tabs)) : tau_old;
  __syncthreads();
  const float tau = c.m->tau;
  compact_buffer(c, [&](float x, int col) { return (col < lo || col >= hi) && x >= tau; });
  const bool ovf = fast_tile(c, t, tau);
  if (__syncthreads_or(ovf) && tid == 0) atomicOr(&c.m->flags, F_OVF);
  __syncthreads();
}

template <int DT>
__device__ void greedy_tile(const Ctx<DT>& c, int t, float& best, int& bidx) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  const uint8_t* st = c.stage(t);
  const int len = c.tile_len(t), lead = c.tile_lead(t);
  const int n_groups = (lead + len + VE - 1) / VE;
  const int colbase = c.c0 + t * TE - lead;
  for (int q = threadIdx.x; q < n_groups; q += kThreads) {
    float x[VE];
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int e = q * VE + i;
      if (e >= lead && e < lead + len && better(x[i], colbase + e, best, bidx)) {
        best = x[i];
        bidx = colbase + e;
      }
    }
  }
  for (int j = c.toff[t] + threadIdx.x; j < c.toff[t + 1]; j += kThreads) {
    const int col = c.c0 + c.bcol[j];
    if (better(c.bx[j], col, best, bidx)) {
      best = c.bx[j];
      bidx = col;
    }
  }
}

__device__ __forceinline__ void hash_insert(int* hkey, int* hcnt, Misc* m, int key, int slots) {
  uint32_t h = (uint32_t(key) * 2654435761u) & uint32_t(slots - 1);
  for (int probe = 0; probe < slots; ++probe) {
    const int prev = atomicCAS(&hkey[h], -1, key);
    if (prev == -1) {
      atomicAdd(&hcnt[h], 1);
      atomicAdd(&m->n_unique, 1);
      return;
    }
    if (prev == key) {
      atomicAdd(&hcnt[h], 1);
      return;
    }
    h = (h + 1) & uint32_t(slots - 1);
  }
  atomicOr(&m->flags, F_HIST);
}

// ---------------------------------------------------------------------------
// block-level helpers for the leader
// ---------------------------------------------------------------------------
__device__ void bitonic_sort_u64(uint64_t* s, int n, bool desc) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += kThreads) {
        const int l = i ^ j;
        if (l > i) {
          const uint64_t a = s[i], b = s[l];
          const bool asc = ((i & k) == 0) != desc;
          if (asc ? (a > b) : (a < b)) {
            s[i] = b;
            s[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Inclusive scan of get(i), i in [0, n), in index order (each thread owns a
// contiguous chunk).  visit(i, inclusive_prefix, total) is called once per i.
template <class Get, class Visit>
__device__ void block_chunk_scan(Misc* m, int n, Get get, Visit visit) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + kThreads - 1) / kThreads;
  const int i0 = min(tid * per, n), i1 = min(i0 + per, n);
  double local = 0.0;
  for (int i = i0; i < i1; ++i) local += get(i);
  double incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) m->d_red[warp] = incl;
  __syncthreads();
  double wbase = 0.0, total = 0.0;
  for (int w = 0; w < kWarps; ++w) {
    if (w < warp) wbase += m->d_red[w];
    total += m->d_red[w];
  }
  double run = wbase + incl - local;
  for (int i = i0; i < i1; ++i) {
    run += get(i);
    visit(i, run, total);
  }
  __syncthreads();
}

__device__ int block_sum_int(Misc* m, int v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  if (lane == 0) m->i_red[warp] = v;
  __syncthreads();
  int s = 0;
  for (int w = 0; w < kWarps; ++w) s += m->i_red[w];
  __syncthreads();
  return s;
}

__device__ __forceinline__ int status_from_flags(int f, bool greedy) {
  if (f & F_TIMEOUT) return NS_ERR_DEVICE_TIMEOUT;
  if (f & F_BADID) return NS_ERR_TOKEN_ID_OUT_OF_RANGE;
  if (f & F_HIST) return NS_ERR_HISTORY_TOO_LONG;
  if (f & F_UNSUP) return NS_ERR_UNSUPPORTED;
  if (greedy) return NS_OK;
  if (f & F_NAN) return NS_ERR_INVALID_DISTRIBUTION;
  if (f & F_OVF) return NS_ERR_CANDIDATE_OVERFLOW;
  return NS_OK;
}

// Leader, FAST rows: survivors sorted by (y desc, id asc); softmax; top-p cut
// (keep sorted j iff j == 0 or cumsum[j-1] <= p, reference sampler.py:122-131);
// then the inverse-CDF draw over the kept ids in ascending id order.
template <int DT>
__device__ void finalize_row(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp) {
  Misc* m = c.m;
  const int tid = threadIdx.x;
  const int n = m->n_merge;
  float* my = reinterpret_cast<float*>(c.stages);
  int* mid = reinterpret_cast<int*>(c.stages + size_t(a.merge_cap) * 4);
  uint64_t* keys = reinterpret_cast<uint64_t*>(c.stages + size_t(a.merge_cap) * 8);
  if (n == 0) {
    if (tid == 0) a.out_ids[row] = NS_ERR_INVALID_DISTRIBUTION;
    return;
  }
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int i = tid; i < n2; i += kThreads)
    keys[i] = (i < n) ? ((uint64_t(f2key(my[i] + 0.0f)) << 32) | uint64_t(~uint32_t(mid[i]))) : 0ull;
  __syncthreads();
  bitonic_sort_u64(keys, n2, true);
  for (int i = tid; i < n; i += kThreads) {
    my[i] = key2f(uint32_t(keys[i] >> 32));
    mid[i] = int(~uint32_t(keys[i]));
  }
  __syncthreads();
  const float M = my[0];
  if (!(M < INFINITY)) {
    if (tid == 0) a.out_ids[row] = NS_ERR_INVALID_DISTRIBUTION;
    return;
  }
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) my[i] = expf(__fsub_rn(my[i], M));
  __syncthreads();
  int L = n;
  if (topp > 0.0f && topp < 1.0f) {
    int cnt = 0;
    const double p = double(topp);
    block_chunk_scan(
        m, n, [&](int i) { return double(my[i]); },
        [&](int i, double incl, double total) { cnt += (i <= n - 2 && incl <= p * total) ? 1 : 0; });
    L = 1 + block_sum_int(m, cnt);
  }
  int n3 = 1;
  while (n3 < L) n3 <<= 1;
  for (int i = tid; i < n3; i += kThreads)
    keys[i] = (i < L) ? ((uint64_t(uint32_t(mid[i])) << 32) | uint64_t(__float_as_uint(my[i]))) : ~0ull;
  __syncthreads();
  bitonic_sort_u64(keys, n3, false);
  const float u = a.uniforms ? a.uniforms[row] : philox_uniform(a.seed, a.offset, uint64_t(row));
  if (tid == 0) m->choose = INT_MAX;
  __syncthreads();
  int first = INT_MAX;
  block_chunk_scan(
      m, L, [&](int i) { return double(__uint_as_float(uint32_t(keys[i]))); },
      [&](int i, double incl, double total) {
        if (first == INT_MAX && incl > double(u) * total) first = i;
      });
  if (first != INT_MAX) atomicMin(&m->choose, first);
  __syncthreads();
  if (tid == 0) {
    const int ch = (m->choose == INT_MAX) ? L - 1 : m->choose;
    a.out_ids[row] = int64_t(uint32_t(keys[ch] >> 32)) + a.vocab_offset;
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const __grid_constant__ KArgs a) {
  using C_ = Ctx<DT>;
  constexpr int TE = C_::TE;
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  const int64_t row = blockIdx.x / CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  C_ c;
  c.stages = smem;
  c.bar = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  c.cx = reinterpret_cast<float*>(smem + a.off_cx);
  c.cid = reinterpret_cast<int*>(smem + a.off_cid);
  c.hist = reinterpret_cast<uint32_t*>(smem + a.off_hist);
  c.hkey = reinterpret_cast<int*>(smem + a.off_hkey);
  c.hcnt = reinterpret_cast<int*>(smem + a.off_hcnt);
  c.bcol = reinterpret_cast<int*>(smem + a.off_bcol);
  c.bcnt = reinterpret_cast<int*>(smem + a.off_bcnt);
  c.bx = reinterpret_cast<float*>(smem + a.off_bx);
  c.toff = reinterpret_cast<int*>(smem + a.off_toff);
  c.tfill = reinterpret_cast<int*>(smem + a.off_tfill);
  c.m = reinterpret_cast<Misc*>(smem + a.off_misc);
  Misc* m = c.m;

  const float T = a.temperature[row];
  const int topk = a.top_k[row];
  const float topp = a.top_p[row];
  const float rep = a.rep ? a.rep[row] : 1.0f;
  const float pres = a.pres ? a.pres[row] : 0.0f;
  const float freq = a.freq ? a.freq[row] : 0.0f;
  int mode;
  if (T == 0.0f)
    mode = MODE_GREEDY;
  else if (topk > 0 && int64_t(topk) < a.vocab_total && topk <= kFastK)
    mode = MODE_FAST;
  else
    mode = MODE_GENERAL;
  c.neg = T < 0.0f;
  c.Tabs = fabsf(T);
  c.K = topk;
  int64_t h0 = 0, h1 = 0;
  if (a.hist_offsets) {
    h0 = a.hist_offsets[row];
    h1 = a.hist_offsets[row + 1];
  }
  const bool pen = (h1 > h0) && (rep != 1.0f || pres != 0.0f || freq != 0.0f);
  c.rowp = reinterpret_cast<const uint8_t*>(a.logits) + size_t(row) * size_t(a.row_stride) * C_::ES;
  c.c0 = int(min(int64_t(rank) * a.per_cta, a.vocab));
  c.c1 = int(min(int64_t(c.c0) + a.per_cta, a.vocab));
  int n_tiles = (c.c1 - c.c0 + TE - 1) / TE;
  if (mode == MODE_GENERAL) n_tiles = 0;
  c.n_tiles = n_tiles;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&c.bar[s], 1);
    fence_mbar_init();
    m->n_cand = 0;
    m->flags = (mode == MODE_GENERAL) ? F_UNSUP : 0;
    m->n_unique = 0;
    m->tau = -INFINITY;
    m->n_merge = 0;
    m->choose = INT_MAX;
    m->g_best = -INFINITY;
    m->g_idx = INT_MAX;
  }
  for (int i = tid; i < a.hash_slots; i += kThreads) {
    c.hkey[i] = -1;
    c.hcnt[i] = 0;
  }
  for (int i = tid; i <= a.tiles_max; i += kThreads) {
    c.toff[i] = 0;
    c.tfill[i] = 0;
  }
  __syncthreads();

  const uint64_t policy = l2_policy_evict_first();
  int issued = 0;  // meaningful in thread 0 only
  if (tid == 0) {
    issued = min(kStages, n_tiles);
    for (int t = 0; t < issued; ++t) issue_tile(c, t, policy);
  }

  // ---- history: distinct in-range ids with counts, bucketed by tile ----
  if (pen && mode != MODE_GENERAL) {
    for (int64_t i = h0 + tid; i < h1; i += kThreads) {
      const int id = a.hist_ids[i];
      if (id < 0 || int64_t(id) >= a.vocab_total) {
        atomicOr(&m->flags, F_BADID);
        continue;
      }
      const int64_t lc = int64_t(id) - a.vocab_offset;
      if (lc >= c.c0 && lc < c.c1) hash_insert(c.hkey, c.hcnt, m, int(lc - c.c0), a.hash_slots);
    }
    __syncthreads();
    if (m->n_unique > a.uniq_cap) {
      if (tid == 0) atomicOr(&m->flags, F_HIST);
    } else if (m->n_unique > 0) {
      for (int i = tid; i < a.hash_slots; i += kThreads)
        if (c.hkey[i] >= 0) atomicAdd(&c.tfill[c.hkey[i] / TE], 1);
      __syncthreads();
      if (warp == 0) {
        int carry = 0;
        for (int base = 0; base < n_tiles; base += 32) {
          const int t = base + lane;
          const int v = (t < n_tiles) ? c.tfill[t] : 0;
          int incl = v;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int w = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += w;
          }
          if (t < n_tiles) {
            c.toff[t] = carry + incl - v;
            c.tfill[t] = 0;
          }
          carry += __shfl_sync(kFull, incl, 31);
        }
        if (lane == 0) c.toff[n_tiles] = carry;
      }
      __syncthreads();
      for (int i = tid; i < a.hash_slots; i += kThreads) {
        const int key = c.hkey[i];
        if (key >= 0) {
          const int t = key / TE;
          const int pos = c.toff[t] + atomicAdd(&c.tfill[t], 1);
          c.bcol[pos] = key;
          c.bcnt[pos] = c.hcnt[i];
        }
      }
    }
    __syncthreads();
  }

  // ---- stream the row ----
  // Per-tile decisions that depend on other warps (a timed-out wait, an
  // overflowing append) are combined with __syncthreads_or so every thread of
  // the CTA takes the same branch.
  float g_best = -INFINITY;
  int g_idx = INT_MAX;
  int t_done = 0;
  bool ovf_local = false;  // this thread's warp overflowed while appending tile t-1
  bool timed_out = false;
  for (int t = 0; t < n_tiles; ++t) {
    const bool ok = mbar_wait_bounded(&c.bar[t % kStages], uint32_t(t / kStages) & 1u);
    if (ok) {
      uint8_t* st = c.stage(t);
      using R = typename Elem<DT>::raw;
      R* sr = reinterpret_cast<R*>(st);
      const int lead = c.tile_lead(t);
      for (int j = c.toff[t] + tid; j < c.toff[t + 1]; j += kThreads) {
        const int e = lead + c.bcol[j] - t * TE;
        float xp = penalize(Elem<DT>::widen(sr[e]), c.bcnt[j], rep, pres, freq);
        if (c.neg) xp = -xp;
        c.bx[j] = xp;
        sr[e] = c.neg ? Elem<DT>::pinf : Elem<DT>::ninf;
      }
      fence_proxy_async_smem();
    }
    bool prev_ovf = false;
    if (__syncthreads_or(!ok || ovf_local)) {
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicOr(&m->flags, F_TIMEOUT);
        timed_out = true;
        break;
      }
      prev_ovf = __syncthreads_or(ovf_local);
    }
    ovf_local = false;
    t_done = t + 1;
    if (mode == MODE_FAST && prev_ovf && !(m->flags & F_OVF)) select_tile(c, t - 1);
    if (tid == 0 && t > 0 && issued < n_tiles) {
      issue_tile(c, issued, policy);
      ++issued;
    }
    if (mode == MODE_GREEDY) {
      greedy_tile(c, t, g_best, g_idx);
    } else if (!(m->flags & F_OVF)) {
      const float tau = m->tau;
      if (tau == -INFINITY && c.tile_len(t) + (c.toff[t + 1] - c.toff[t]) > kCap / 2)
        select_tile(c, t);
      else
        ovf_local = fast_tile(c, t, tau);
    }
  }
  const bool last_ovf = __syncthreads_or(ovf_local);
  // After a timeout, wait (bounded) for copies still in flight before the
  // shared memory is reused or released.
  if (tid == 0) {
    for (int t = t_done; t < issued; ++t) mbar_wait_bounded(&c.bar[t % kStages], uint32_t(t / kStages) & 1u);
  }
  __syncthreads();

  if (mode == MODE_FAST && !timed_out && !(m->flags & F_OVF)) {
    if (last_ovf) select_tile(c, n_tiles - 1);
    if (!(m->flags & F_OVF) && m->n_cand > c.K) {
      const int n = m->n_cand;
      uint32_t key = 0;
      const bool have = radix_kth(
          c, c.K,
          [&](auto f) {
            for (int i = tid; i < n; i += kThreads) f(c.cx[i]);
          },
          &key);
      if (tid == 0 && have) m->tau = fmaxf(m->tau, scaled_lower_bound(key2f(key), c.Tabs));
      __syncthreads();
      const float tau = m->tau;
      compact_buffer(c, [&](float x, int) { return x >= tau; });
    }
  }
  if (mode == MODE_GREEDY) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(kFull, g_best, o);
      const int oi = __shfl_xor_sync(kFull, g_idx, o);
      if (better(ob, oi, g_best, g_idx)) {
        g_best = ob;
        g_idx = oi;
      }
    }
    if (lane == 0) {
      m->f_red[warp] = g_best;
      m->i_red[warp] = g_idx;
    }
    __syncthreads();
    if (tid == 0) {
      float b = m->f_red[0];
      int bi = m->i_red[0];
      for (int w = 1; w < kWarps; ++w)
        if (better(m->f_red[w], m->i_red[w], b, bi)) {
          b = m->f_red[w];
          bi = m->i_red[w];
        }
      m->g_best = b;
      m->g_idx = bi;
    }
  }
  __syncthreads();

  // ---- cluster merge ----
  cluster.sync();
  if (rank == 0) {
    if (tid == 0) {
      int fl = 0, tot = 0;
      float b = -INFINITY;
      int bi = INT_MAX;
      for (int r = 0; r < CL; ++r) {
        Misc* rm = cluster.map_shared_rank(m, r);
        fl |= rm->flags;
        m->roff[r] = tot;
        m->rc0[r] = int(min(int64_t(r) * a.per_cta, a.vocab));
        tot += rm->n_cand;
        if (better(rm->g_best, rm->g_idx, b, bi)) {
          b = rm->g_best;
          bi = rm->g_idx;
        }
      }
      m->roff[CL] = tot;
      m->flags = fl;
      if (mode == MODE_GREEDY) {
        const int st = status_from_flags(fl, true);
        a.out_ids[row] = (st != NS_OK) ? int64_t(st) : int64_t(bi) + a.vocab_offset;
      } else if (status_from_flags(fl, false) != NS_OK) {
        a.out_ids[row] = status_from_flags(fl, false);
      }
    }
    __syncthreads();
    if (mode == MODE_FAST && status_from_flags(m->flags, false) == NS_OK) {
      const int tot = m->roff[CL];
      auto owner = [&](int gi) {
        int r = 0;
        while (r + 1 < CL && m->roff[r + 1] <= gi) ++r;
        return r;
      };
      uint32_t key = 0;
      const bool have = (tot > c.K) && radix_kth(
                                           c, c.K,
                                           [&](auto f) {
                                             for (int gi = tid; gi < tot; gi += kThreads) {
                                               const int r = owner(gi);
                                               const float* rcx = cluster.map_shared_rank(c.cx, r);
                                               f(rcx[gi - m->roff[r]]);
                                             }
                                           },
                                           &key);
      const float thr = have ? __fdiv_rn(key2f(key), c.Tabs) : -INFINITY;
      float* my = reinterpret_cast<float*>(c.stages);
      int* mid = reinterpret_cast<int*>(c.stages + size_t(a.merge_cap) * 4);
      for (int gi = tid; gi < tot; gi += kThreads) {
        const int r = owner(gi);
        const float* rcx = cluster.map_shared_rank(c.cx, r);
        const int* rcid = cluster.map_shared_rank(c.cid, r);
        const float y = __fdiv_rn(rcx[gi - m->roff[r]], c.Tabs);
        if (y >= thr) {
          const int pos = atomicAdd(&m->n_merge, 1);
          if (pos < a.merge_cap) {
            my[pos] = y;
            mid[pos] = rcid[gi - m->roff[r]] + m->rc0[r];
          }
        }
      }
      __syncthreads();
      if (tid == 0 && m->n_merge > a.merge_cap) {
        m->flags |= F_OVF;
        a.out_ids[row] = NS_ERR_CANDIDATE_OVERFLOW;
      }
      __syncthreads();
    }
  }
  cluster.sync();
  if (rank == 0 && mode == MODE_FAST && status_from_flags(m->flags, false) == NS_OK) finalize_row(c, a, row, topp);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  uint32_t off_bar, off_cx, off_cid, off_hist, off_hkey, off_hcnt, off_bcol, off_bcnt, off_bx, off_toff,
      off_tfill, off_misc, total;
};

static uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

static Layout make_layout(int hash_slots, int uniq_cap, int tiles_max) {
  Layout L;
  uint32_t o = kStages * kStageStride;
  L.off_bar = o;
  o += kStages * 8;
  o = align_up(o, 16);
  L.off_cx = o;
  o += kCap * 4;
  L.off_cid = o;
  o += kCap * 4;
  L.off_hist = o;
  o += kBins * 4;
  L.off_hkey = o;
  o += hash_slots * 4;
  L.off_hcnt = o;
  o += hash_slots * 4;
  L.off_bcol = o;
  o += uniq_cap * 4;
  L.off_bcnt = o;
  o += uniq_cap * 4;
  L.off_bx = o;
  o += uniq_cap * 4;
  L.off_toff = o;
  o += (tiles_max + 1) * 4;
  L.off_tfill = o;
  o += (tiles_max + 1) * 4;
  o = align_up(o, 16);
  L.off_misc = o;
  o += sizeof(Misc);
  L.total = align_up(o, 128);
  return L;
}

struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;
  uint32_t configured[3] = {0, 0, 0};
};

static std::mutex g_mu;
static DeviceInfo g_dev[64];

template <int DT>
static int launch(const KArgs& base, int64_t batch, ns_stream_t stream) {
  using C_ = Ctx<DT>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NS_ERR_CUDA;
  DeviceInfo* di = &g_dev[dev];
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (di->sms == 0) {
      if (cudaDeviceGetAttribute(&di->sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return NS_ERR_CUDA;
      if (cudaDeviceGetAttribute(&di->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
          cudaSuccess)
        return NS_ERR_CUDA;
    }
  }
  KArgs a = base;
  const int64_t V = a.vocab;
  // CTAs per row: enough rows x CTAs to cover the SMs, each CTA >= 2 tiles.
  int CL = 1;
  while (CL < kMaxCluster && batch * CL < di->sms && V / (2 * CL) >= C_::TE) CL *= 2;
  int64_t per = (V + CL - 1) / CL;
  per = (per + C_::VE - 1) / C_::VE * C_::VE;
  a.per_cta = int(per);
  a.tiles_max = int((per + C_::TE - 1) / C_::TE);
  int64_t hmax = 0;
  if (a.hist_ids) hmax = std::min<int64_t>(a.max_history, per);
  int slots = 32;
  while (slots < 2 * hmax && slots < kHashMax) slots <<= 1;
  a.hash_slots = slots;
  a.uniq_cap = int(std::min<int64_t>(std::max<int64_t>(hmax, 1), slots));
  const Layout L = make_layout(a.hash_slots, a.uniq_cap, a.tiles_max);
  a.merge_cap = 1;
  while (a.merge_cap * 2 * 16 <= kStages * kStageStride) a.merge_cap <<= 1;
  a.off_bar = L.off_bar;
  a.off_cx = L.off_cx;
  a.off_cid = L.off_cid;
  a.off_hist = L.off_hist;
  a.off_hkey = L.off_hkey;
  a.off_hcnt = L.off_hcnt;
  a.off_bcol = L.off_bcol;
  a.off_bcnt = L.off_bcnt;
  a.off_bx = L.off_bx;
  a.off_toff = L.off_toff;
  a.off_tfill = L.off_tfill;
  a.off_misc = L.off_misc;
  if (int(L.total) > di->max_smem_optin) return NS_ERR_INVALID_ARGUMENT;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (di->configured[DT] < L.total) {
      if (cudaFuncSetAttribute(sample_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L.total)) !=
          cudaSuccess)
        return NS_ERR_CUDA;
      di->configured[DT] = L.total;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(batch * CL), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(CL);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, sample_kernel<DT>, a) != cudaSuccess) return NS_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return NS_ERR_CUDA;
  return NS_OK;
}

}  // namespace ns

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

const char* ns_status_string(int status) {
  switch (status) {
    case NS_OK: return "ok";
    case NS_ERR_INVALID_ARGUMENT: return "invalid argument";
    case NS_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case NS_ERR_UNSUPPORTED_DTYPE: return "unsupported logits dtype";
    case NS_ERR_CUDA: return "CUDA error";
    case NS_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case NS_ERR_TOKEN_ID_OUT_OF_RANGE: return "history token id out of range";
    case NS_ERR_INVALID_DISTRIBUTION:
      return "probability tensor contains either `inf`, `nan` or element < 0";
    case NS_ERR_HISTORY_TOO_LONG: return "too many distinct history ids for one block";
    case NS_ERR_CANDIDATE_OVERFLOW: return "ties at the top-k threshold exceed the candidate buffers";
    case NS_ERR_UNSUPPORTED: return "unsupported parameter combination";
    default: return "unknown status";
  }
}

int ns_version(void) { return 100; }

int ns_sampler_workspace_bytes(int64_t batch, int64_t vocab, int64_t max_history, size_t* out_bytes) {
  if (!out_bytes || batch < 0 || vocab <= 0 || max_history < 0) return NS_ERR_INVALID_ARGUMENT;
  *out_bytes = 0;
  return NS_OK;
}

int ns_sample(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
              const int32_t* hist_ids, const int64_t* hist_offsets, int64_t max_history,
              const float* temperature, const int32_t* top_k, const float* top_p,
              const float* repetition_penalty, const float* presence_penalty, const float* frequency_penalty,
              const float* uniforms, uint64_t philox_seed, uint64_t philox_offset, int64_t* out_ids,
              void* workspace, size_t workspace_bytes, ns_stream_t stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (dtype != NS_DTYPE_F32 && dtype != NS_DTYPE_BF16 && dtype != NS_DTYPE_F16) return NS_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || vocab <= 0 || row_stride < vocab || max_history < 0) return NS_ERR_INVALID_ARGUMENT;
  if (vocab > (int64_t(1) << 30) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
  if ((hist_ids == nullptr) != (hist_offsets == nullptr)) return NS_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NS_OK;
  if (!logits || !temperature || !top_k || !top_p || !out_ids) return NS_ERR_INVALID_ARGUMENT;
  ns::KArgs a = {};
  a.logits = logits;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.vocab_offset = 0;
  a.vocab_total = vocab;
  a.hist_ids = hist_ids;
  a.hist_offsets = hist_offsets;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.rep = repetition_penalty;
  a.pres = presence_penalty;
  a.freq = frequency_penalty;
  a.uniforms = uniforms;
  a.seed = philox_seed;
  a.offset = philox_offset;
  a.out_ids = out_ids;
  a.max_history = max_history;
  switch (dtype) {
    case NS_DTYPE_F32: return ns::launch<NS_DTYPE_F32>(a, batch, stream);
    case NS_DTYPE_BF16: return ns::launch<NS_DTYPE_BF16>(a, batch, stream);
    default: return ns::launch<NS_DTYPE_F16>(a, batch, stream);
  }
}

}  // extern "C"
