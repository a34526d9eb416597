// B200-native token sampler (sm_100a).
//
// One launch samples every row of a batch.  Each row is handled by one CTA
// (256 threads), or by a thread block cluster of up to 8 CTAs when the batch
// is too small to fill the SMs; CTA r owns columns [r*per_cta, (r+1)*per_cta)
// of the row, and each of its 8 warps owns a contiguous 1/8 of that range.  A
// warp streams its columns once from HBM through its own 2-stage ring of 4 KB
// bulk copies (TMA, cp.async.bulk) into shared memory and consumes them with
// no block-wide barrier: its threshold, candidate buffer and argmax live in
// warp-uniform registers and warp-private shared memory.  Block (and cluster)
// synchronisation happens at the seed and at the end of the row.  Per row, by
// mode:
//
//   GREEDY (temperature == 0; reference sampler.py:60-70)
//       first-index argmax of the penalised logits (NaN counts as max).
//   FAST   (0 < top_k <= kFastK; reference sampler.py:73-89, 110-133)
//       single-pass threshold filter: each warp keeps every value >= tau, a
//       lower bound of the CTA's k-th largest shared between the warps without
//       barriers; the survivors of the tightest bound are sorted as 64-bit keys
//       (scaled value, id), and the top-k with ties, top-p and the inverse-CDF
//       draw run on them.  The vocabulary is never sorted.
//   SOFTMAX (top-k and top-p both off -- the reference's defaults)
//       one pass of per-tile maxima and float64 masses; the draw is located by
//       CTA (clusters exchange maxima and masses), warp, then tile, and one
//       4 KB tile is read again.
//   NUCLEUS (top-k off, top-p on)
//       FAST with the kNucleusK largest as candidates plus the SOFTMAX masses;
//       when the candidates hold more than p of the row's mass, the top-p cut
//       and the draw run on them; otherwise (one CTA per row) one more pass
//       collects a window of values below the row's maximum (nucleus_wide),
//       else GENERAL.
//   WIDEK  (kWideKFrom <= top_k <= kWideCap, one CTA per row)
//       FAST with kNucleusK candidates, then one more pass counting and
//       collecting the values in a window below the row's maximum
//       (wide_topk), else GENERAL.
//   GENERAL (top-k beyond those, ties overflowing a buffer, NUCLEUS rows whose
//       nucleus is larger)
//       a cluster-cooperative multi-pass radix search over counts and
//       fixed-point masses; the last pass rescans one tile in id order.
//
// Penalties (reference sampler.py:93-108 plus presence/frequency): before the
// stream starts, each CTA sets a column bitmap from the row's history ids,
// ranks the distinct ids in column order and counts their occurrences (shared
// atomics without return values).  When a tile lands, its history slots --
// one rank range -- have their raw values recorded and are overwritten with
// -inf so the streaming passes see only un-penalised columns; after its last
// tile each warp penalises its recorded values in fp32 (IEEE division /
// multiplication / subtraction, never contracted into FMAs) and adds them once.
//
// Temperature is applied without a per-element division on the FAST path: y
// = x / T is monotone in x, so the survivors {rn(x / T) >= rn(x_k / T)} are
// {x >= x_lo} for the smallest x_lo with rn(x_lo / T) >= rn(x_k / T) (found by
// a short search over float keys, or bounded from below without divisions).
// Negative temperatures are handled by negating x (rn(-x / -T) = rn(x / T)).
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>
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
constexpr int kWTile = 4096;                    // bytes per warp tile
constexpr int kWStages = 2;                     // per-warp ring depth
constexpr int kWStageStride = kWTile + 32;      // + alignment lead + vector overrun
constexpr int kStageBytes = kWarps * kWStages * kWStageStride;
constexpr int kCapW = 256;                      // per-warp candidate buffer (entries)
constexpr int kPerLane = kCapW / 32;
constexpr int kFastK = 240;                     // largest top_k served by the single-pass path
constexpr int kWideKFrom = 225;                 // one-CTA rows from this top_k on take WIDEK: near kFastK
                                                // the warps' candidate buffers overflow on some rows
constexpr int kNucleusK = 128;                  // NUCLEUS candidates (the largest values with ties)
static_assert((kFastK + kWarps - 1) / kWarps <= 32, "a warp's published rank is one of its 32 lane maxima");
constexpr int kCandBytes = kWarps * kCapW * 8;  // candidate buffers (x, col)
constexpr int kBins = 256;                      // radix digit = 8 bits (one bin per thread)
static_assert(kBins == kThreads, "block_kth_regs clears one bin per thread");
constexpr int kMaxCluster = 8;
// leader merge area in the stage bytes: y[] and id[] lists, then u64 sort keys
constexpr int kMergeCap = 4096;
static_assert(kMergeCap * 16 <= kStageBytes, "merge lists and their sort keys fit the stage area");
constexpr int kMaxLists = kMaxCluster * kWarps;
// Distinct history ids one CTA keeps in shared memory (12 B each: count,
// column, penalised value).  A CTA whose columns hold more moves its rank
// arrays to the caller's workspace, so shared memory does not grow with the
// history length.
constexpr int kHistSmem = 1024;
constexpr unsigned kFull = 0xFFFFFFFFu;

enum : int { MODE_GREEDY = 0, MODE_FAST = 1, MODE_GENERAL = 2, MODE_SOFTMAX = 3, MODE_NUCLEUS = 4, MODE_WIDEK = 5 };
enum : int { F_NAN = 1, F_BADID = 2, F_HIST = 4, F_OVF = 8, F_TIMEOUT = 16, F_UNSUP = 32, F_BIG = 64 };

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
  int flags;      // F_* bits of this CTA (the leader's becomes the cluster's)
  int r_digit;    // radix-select broadcast
  int r_krem;
  int n_merge;    // leader: survivors gathered from the cluster
  int choose;     // leader: inverse-CDF pick
  float g_best;   // greedy result of this CTA
  int g_idx;      // ... as a column of this call's logits
  int wn[kWarps];  // per-warp candidate counts after streaming
  float wbest[kWarps];
  int widx[kWarps];
  double d_red[kWarps];
  int i_red[kWarps];
  // GENERAL rows (cluster-cooperative multi-pass)
  unsigned g_maxk;              // this CTA's max key of x (finite values)
  int g_bin;                    // digit search: crossing bin (-1: none)
  unsigned long long g_before;  // digit search: cumulative value above the crossing bin
  unsigned long long g_mass;    // this CTA's (kept) mass, fixed point
  unsigned long long g_sum[kWarps];
  int g_ties;                   // this CTA's count of values equal to the top-p cut
  int g_tile;                   // inverse CDF: chosen tile of this CTA (-1: none)
  unsigned long long g_tbefore; // ... and the kept mass before it
  int segoff[kWarps + 1];   // distinct history ids before each warp's columns
  uint32_t pub[kWarps];     // FAST: per-warp published bound (key; 0 = none)
  double s_rem;             // SOFTMAX: the draw's remaining mass inside the chosen warp
  int s_warp;               // ... and that warp
  int s_rank;               // ... and that CTA of the cluster
  int hist_g;               // the rank arrays live in the workspace (more than cnt_cap distinct ids)
  float c_M;                // SOFTMAX clusters: this CTA's largest scaled value
  double c_W;               // ... and its mass with the row's largest
  float nuc_M;              // NUCLEUS: the row's largest scaled value
  double nuc_Z;             // ... and its total mass sum exp(y - nuc_M)
  float nuc_yk;             // ... and its kNucleusK-th largest scaled value (-inf: unknown)
  float nuc_cov;            // ... and the share of the mass those hold (-1: unknown)
  int w_bin;                // wide NUCLEUS: last bin of the candidate set
  int w_n;                  // ... its count, and the keys collected
  int w_tot;                // ... values counted in the window
  int w_binb;               // large nucleus: the bin where the exact mass crosses p Z
  int w_cntb;               // ... and its count
  unsigned long long w_keyL;  // large nucleus: the last kept key of the boundary bin
  int w_L;                  // ... and how many of its keys are kept (-1: none / fall back)
  int roff[kMaxLists + 1];  // leader: union offsets over (rank, warp) lists
  int rc0[kMaxCluster];     // leader: first column of each rank
  uint32_t hist[kBins];
};

struct KArgs {
  const void* logits;
  int64_t vocab;         // columns read per row
  int64_t row_stride;    // elements between rows
  int64_t vocab_offset;  // global id of column 0 (vocab-parallel slices)
  int64_t vocab_total;   // global vocabulary size
  const int32_t* hist_ids;
  const int64_t* hist_offsets;
  int64_t max_history;
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
  int per_cta;     // columns per CTA (multiple of the 16-byte vector width)
  int per_warp;    // columns per warp (multiple of the 16-byte vector width)
  int tpw;         // tiles per warp (upper bound)
  int nwords;      // history bitmap words (one bit per column of a CTA)
  int cnt_cap;     // distinct history ids the shared-memory rank arrays hold
  // rank arrays of CTAs with more distinct ids (nullptr: none): per CTA
  // hist_ws_cap counts, then columns, then penalised values
  int32_t* hist_ws;
  int hist_ws_cap;
  void* ws;         // the caller's workspace and its size
  size_t ws_bytes;
  int merge_cap;   // leader merge area (entries)
  // vocab-parallel local step: out_ids[] receives each row's survivor count
  // (or a negative status) and vp_keys[row * vp_cap ...] its sorted keys
  int64_t* vp_keys;
  int vp_cap;
  uint32_t off_bar, off_cand, off_bits, off_pre, off_cnt, off_colr, off_pval, off_tacc, off_misc;
};

template <int DT>
struct Ctx {
  using E = Elem<DT>;
  static constexpr int ES = E::size;
  static constexpr int VE = 16 / ES;      // elements per 16-byte vector
  static constexpr int TE = kWTile / ES;  // elements per warp tile

  uint8_t* stages;
  uint64_t* bar;
  float* cx;  // [kWarps][kCapW]
  int* cid;   // [kWarps][kCapW]
  uint32_t* bits;  // history membership, one bit per CTA column
  uint16_t* pre;   // set bits of the owning warp's columns before each word
  int* cnt;        // occurrences of each distinct history id, by rank
  int* colr;       // CTA-relative column of each distinct history id, by rank
  float* pval;     // its penalised value (negated when T < 0), by rank
  void* tacc;
  Misc* m;

  const uint8_t* rowp;  // column 0 of this row
  int64_t row;
  int c0, c1;           // this CTA's columns
  int pw, tpw;          // per-warp columns / tiles
  int nwords;
  int K;
  bool neg;
  bool pen;  // this row has a history and a non-neutral penalty
  float Tabs;
  float rep, pres, freq;
  float u_pre;  // the row's caller-supplied uniform (loaded when the kernel starts)

  __device__ __forceinline__ int w0(int w) const { return min(c0 + w * pw, c1); }
  __device__ __forceinline__ int w1(int w) const { return min(c0 + (w + 1) * pw, c1); }
  __device__ __forceinline__ int wtiles(int w) const { return (w1(w) - w0(w) + TE - 1) / TE; }
  __device__ __forceinline__ int tile_len(int w, int t) const { return min(TE, w1(w) - (w0(w) + t * TE)); }
  // Elements before the first 16-byte aligned column of a tile; the tile's
  // first column goes to shared-memory slot `lead` so the aligned body lands
  // on a 16-byte boundary.
  __device__ __forceinline__ int tile_head(int w, int t) const {
    const uintptr_t a = reinterpret_cast<uintptr_t>(rowp) + uintptr_t(w0(w) + t * TE) * ES;
    return min(int(((16u - (a & 15u)) & 15u) / ES), tile_len(w, t));
  }
  __device__ __forceinline__ int tile_lead(int w, int t) const { return (VE - tile_head(w, t)) % VE; }
  __device__ __forceinline__ uint8_t* stage(int w, int s) const {
    return stages + (w * kWStages + s) * kWStageStride;
  }
  __device__ __forceinline__ uint64_t* sbar(int w, int s) const { return bar + w * kWStages + s; }
  // Rank (distinct history ids before it, in column order) of CTA-relative
  // column col, a multiple of 32 inside warp w's columns.
  __device__ __forceinline__ int rank_at(int w, int col) const { return m->segoff[w] + pre[col >> 5]; }
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

// A filter bound at or below scaled_lower_bound(xk, T) without divisions: if
// x <= xk - |xk| 2^-21 then x / T lies below xk / T by more than two relative
// rounding errors (2^-24 each in the normal range), so rn(x / T) <
// rn(xk / T).  xk - |xk| 2^-20 is below that even after its own rounding.
// Magnitudes where x / T could leave the normal range use the exact search.
__device__ __forceinline__ float fast_lower_bound(float xk, float T) {
  const float a = fabsf(xk);
  if (a >= 0x1p-60f && a <= 0x1p60f && T >= 0x1p-30f && T <= 0x1p30f) return fmaf(-a, 0x1p-20f, xk);
  return scaled_lower_bound(xk, T);
}

// ---------------------------------------------------------------------------
// per-warp candidate buffer (warp-uniform state)
// ---------------------------------------------------------------------------
struct WarpCand {
  float* x;    // this warp's kCapW-entry buffer
  int* col;
  float tau;   // filter threshold
  int n;       // entries in use
  bool ovf;    // ties exceeded the buffer
};

// K-th largest key among this warp's buffer entries (n > K): bitwise radix
// select over registers, one warp reduction per bit.
__device__ __forceinline__ uint32_t warp_kth_key(const uint32_t (&key)[kPerLane], int K) {
  uint32_t pre = 0;
#pragma unroll 1
  for (int b = 31; b >= 0; --b) {
    const uint32_t cand = pre | (1u << b);
    int cnt = 0;
#pragma unroll
    for (int q = 0; q < kPerLane; ++q) cnt += (key[q] >= cand) ? 1 : 0;
    cnt = int(__reduce_add_sync(kFull, unsigned(cnt)));
    if (cnt >= K) pre = cand;
  }
  return pre;
}

// Raise tau to the collision-safe bound of the warp's K-th largest entry and
// drop the entries below it.
template <int DT>
__device__ void warp_compact(const Ctx<DT>& c, WarpCand& s) {
  const int lane = threadIdx.x & 31;
  uint32_t key[kPerLane];
  int col[kPerLane];
#pragma unroll
  for (int q = 0; q < kPerLane; ++q) {
    const int i = q * 32 + lane;
    key[q] = (i < s.n) ? f2key(s.x[i]) : 0u;
    col[q] = (i < s.n) ? s.col[i] : 0;
  }
  __syncwarp();
  if (s.n > c.K) {
    const uint32_t kk = warp_kth_key(key, c.K);
    float t = 0.0f;
    if (lane == 0) t = fast_lower_bound(key2f(kk), c.Tabs);
    s.tau = fmaxf(s.tau, __shfl_sync(kFull, t, 0));
  }
  int base = 0;
#pragma unroll
  for (int q = 0; q < kPerLane; ++q) {
    const int i = q * 32 + lane;
    const float v = key2f(key[q]);
    const bool keep = (i < s.n) && v >= s.tau;
    const unsigned mk = __ballot_sync(kFull, keep);
    if (keep) {
      const int pos = base + __popc(mk & lanemask_lt());
      s.x[pos] = v;
      s.col[pos] = col[q];
    }
    base += __popc(mk);
  }
  s.n = base;
  __syncwarp();
}

// Drop the warp's buffer entries below tau (after tau was raised elsewhere).
__device__ __forceinline__ void warp_drop_below(WarpCand& s) {
  const int lane = threadIdx.x & 31;
  float v[kPerLane];
  int col[kPerLane];
#pragma unroll
  for (int q = 0; q < kPerLane; ++q) {
    const int i = q * 32 + lane;
    v[q] = (i < s.n) ? s.x[i] : -INFINITY;
    col[q] = (i < s.n) ? s.col[i] : 0;
  }
  __syncwarp();
  int base = 0;
#pragma unroll
  for (int q = 0; q < kPerLane; ++q) {
    const bool keep = (q * 32 + lane < s.n) && v[q] >= s.tau;
    const unsigned mk = __ballot_sync(kFull, keep);
    if (keep) {
      const int pos = base + __popc(mk & lanemask_lt());
      s.x[pos] = v[q];
      s.col[pos] = col[q];
    }
    base += __popc(mk);
  }
  s.n = base;
  __syncwarp();
}

// Warp-wide append: lane l contributes the elements x[i] whose bit i is set
// in `bits`, at columns col0 + i.  All 32 lanes call it.  Compacts first when
// the entries do not fit; a buffer still full afterwards (ties at the
// threshold) sets s.ovf.
template <int DT, int N>
__device__ __forceinline__ void warp_append_bits(const Ctx<DT>& c, WarpCand& s, unsigned bits, const float (&x)[N],
                                                 int col0) {
  const int lane = threadIdx.x & 31;
  int cnt = __popc(bits);
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  int total = __shfl_sync(kFull, incl, 31);
  if (total == 0) return;
  if (s.n + total > kCapW) {
    warp_compact(c, s);
    unsigned nb = 0;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (((bits >> i) & 1u) && x[i] >= s.tau) nb |= 1u << i;
    bits = nb;
    cnt = __popc(bits);
    incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    total = __shfl_sync(kFull, incl, 31);
    if (s.n + total > kCapW) {
      s.ovf = true;
      return;
    }
  }
  int pos = s.n + incl - cnt;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if ((bits >> i) & 1u) {
      s.x[pos] = x[i];
      s.col[pos] = col0 + i;
      ++pos;
    }
  s.n += total;
}

// ---------------------------------------------------------------------------
// producer: one bulk copy per warp tile (plain loads for an unaligned head /
// tail); issued by lane 0 of the owning warp
// ---------------------------------------------------------------------------
template <int DT>
__device__ __forceinline__ void issue_full_tile(const Ctx<DT>& c, int w, int t, int s, uint64_t policy) {
  const uint8_t* src = c.rowp + size_t(c.w0(w) + t * Ctx<DT>::TE) * Ctx<DT>::ES;
  mbar_arrive_expect_tx(c.sbar(w, s), kWTile);
  bulk_g2s(c.stage(w, s), src, kWTile, c.sbar(w, s), policy);
}

template <int DT>
__device__ void issue_tile(const Ctx<DT>& c, int w, int t, int s, uint64_t policy) {
  using E = Elem<DT>;
  constexpr int ES = E::size;
  const int len = c.tile_len(w, t);
  const int head = c.tile_head(w, t);
  const int body = (((len - head) * ES) & ~15) / ES;
  const int tail = len - head - body;
  const int lead = c.tile_lead(w, t);
  const typename E::raw* src = reinterpret_cast<const typename E::raw*>(c.rowp) + (c.w0(w) + t * Ctx<DT>::TE);
  typename E::raw* d = reinterpret_cast<typename E::raw*>(c.stage(w, s));
  for (int q = 0; q < head; ++q) d[lead + q] = src[q];
  for (int q = 0; q < tail; ++q) d[lead + head + body + q] = src[head + body + q];
  const uint32_t bytes = uint32_t(body) * ES;
  mbar_arrive_expect_tx(c.sbar(w, s), bytes);
  if (bytes) bulk_g2s(d + lead + head, src + head, bytes, c.sbar(w, s), policy);
}

// History columns of warp tile (w, t).  The prologue stored each distinct
// history column of the CTA at its rank (history columns before it): colr[]
// its CTA-relative column, pval[] its penalised value (negated when T < 0).
// Ranks follow column order, so a tile's history columns are one rank range.
template <int DT>
__device__ __forceinline__ int2 tile_ranks(const Ctx<DT>& c, int w, int t) {
  constexpr int TE = Ctx<DT>::TE;
  const int base = w * c.pw + t * TE;  // a multiple of 32
  const int r0 = c.rank_at(w, base);
  const int r1 = (t + 1 < c.wtiles(w)) ? c.rank_at(w, base + TE) : c.m->segoff[w + 1];
  return make_int2(r0, r1);
}

// Penalise the history columns of a landed tile: each value is computed from
// its slot and its occurrence count, stored at its rank in pval[] and passed
// to emit(has, x, col) -- called by all 32 lanes once per round of 32
// entries, `has` false for idle lanes, col relative to the CTA's first column
// -- and the slot becomes -inf so passes over the raw slots skip it.
template <int DT, class Emit>
__device__ __forceinline__ void patch_tile(const Ctx<DT>& c, int w, int t, uint8_t* st, Emit emit) {
  using E = Elem<DT>;
  using R = typename E::raw;
  if (!c.pen) return;
  const int lane = threadIdx.x & 31;
  const int2 rr = tile_ranks(c, w, t);
  if (rr.y <= rr.x) return;
  const int base = w * c.pw + t * Ctx<DT>::TE;
  const int lead = c.tile_lead(w, t);
  R* sr = reinterpret_cast<R*>(st);
  for (int r = rr.x; r < rr.y; r += 32) {
    const int ri = r + lane;
    const bool has = ri < rr.y;
    float xp = 0.0f;
    int col = 0;
    if (has) {
      col = c.colr[ri];
      const int e = lead + (col - base);
      xp = penalize(E::widen(sr[e]), c.cnt[ri], c.rep, c.pres, c.freq);
      if (c.neg) xp = -xp;
      c.pval[ri] = xp;
      sr[e] = c.neg ? E::pinf : E::ninf;
    }
    emit(has, xp, col);
  }
  fence_proxy_async_smem();  // the slots are rewritten by a later bulk copy
}

// Streaming passes: the history slots become -inf and their raw values go to
// pval[]; penalize_segment() turns them into penalised values once the warp's
// tiles are done.
template <int DT>
__device__ __forceinline__ void mask_tile(const Ctx<DT>& c, int w, int t, uint8_t* st) {
  using E = Elem<DT>;
  using R = typename E::raw;
  if (!c.pen) return;
  const int lane = threadIdx.x & 31;
  const int2 rr = tile_ranks(c, w, t);
  if (rr.y <= rr.x) return;
  const int base = w * c.pw + t * Ctx<DT>::TE;
  const int lead = c.tile_lead(w, t);
  R* sr = reinterpret_cast<R*>(st);
  for (int ri = rr.x + lane; ri < rr.y; ri += 32) {
    const int e = lead + (c.colr[ri] - base);
    c.pval[ri] = E::widen(sr[e]);
    sr[e] = c.neg ? E::pinf : E::ninf;
  }
  fence_proxy_async_smem();  // the slots are rewritten by a later bulk copy
}

// Penalise the raw values mask_tile() recorded for warp w's columns.
template <int DT>
__device__ __forceinline__ void penalize_segment(const Ctx<DT>& c, int w) {
  const int lane = threadIdx.x & 31;
  for (int r = c.m->segoff[w] + lane; r < c.m->segoff[w + 1]; r += 32) {
    const float x = penalize(c.pval[r], c.cnt[r], c.rep, c.pres, c.freq);
    c.pval[r] = c.neg ? -x : x;
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------
// per-warp streaming passes
// ---------------------------------------------------------------------------
// Load 16-byte group q of a landed tile as fp32 (negated when NEG); groups
// past the tile read as -inf.
template <int DT, bool NEG>
__device__ __forceinline__ void load_group(const uint8_t* st, int q, int n_groups, float (&x)[Ctx<DT>::VE]) {
  if (q < n_groups) {
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
    if (NEG) {
#pragma unroll
      for (int i = 0; i < Ctx<DT>::VE; ++i) x[i] = -x[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < Ctx<DT>::VE; ++i) x[i] = -INFINITY;
  }
}

// Bits of the group's elements that pass the filter (x >= tau); elements
// outside the tile are masked.  NaN or +inf in a sampled row flags F_NAN.
template <int DT>
__device__ __forceinline__ unsigned group_bits(const Ctx<DT>& c, const WarpCand& s, int q,
                                               const float (&x)[Ctx<DT>::VE], int lead, int len, int n_groups) {
  constexpr int VE = Ctx<DT>::VE;
  unsigned bits = 0, bad = 0;
#pragma unroll
  for (int i = 0; i < VE; ++i) {
    bits |= (x[i] >= s.tau ? 1u : 0u) << i;
    bad |= (x[i] != x[i] || x[i] == INFINITY) ? 1u : 0u;
  }
  const int e0 = q * VE;
  if (q >= n_groups || e0 < lead || e0 + VE > lead + len) {  // partial group: mask by position
    unsigned vm = 0;
#pragma unroll
    for (int i = 0; i < VE; ++i) vm |= ((q < n_groups && e0 + i >= lead && e0 + i < lead + len) ? 1u : 0u) << i;
    bits &= vm;
    if (bad) {
      bad = 0;
#pragma unroll
      for (int i = 0; i < VE; ++i) bad |= (((vm >> i) & 1u) && (x[i] != x[i] || x[i] == INFINITY)) ? 1u : 0u;
    }
  }
  if (bad) {
    atomicOr(&c.m->flags, F_NAN);
#pragma unroll
    for (int i = 0; i < VE; ++i)
      if (x[i] != x[i] || x[i] == INFINITY) bits &= ~(1u << i);
  }
  if (s.tau == -INFINITY) {  // no threshold yet: -inf never becomes a candidate
#pragma unroll
    for (int i = 0; i < VE; ++i)
      if (!(x[i] > -INFINITY)) bits &= ~(1u << i);
  }
  return bits;
}

// Append one hot group per lane: the common case (every lane has at most one
// passing element) is a ballot; otherwise the general scan.
template <int DT>
__device__ __forceinline__ void group_append(const Ctx<DT>& c, WarpCand& s, int q, const float (&x)[Ctx<DT>::VE],
                                             bool lane_hot, int lead, int len, int n_groups, int colbase) {
  constexpr int VE = Ctx<DT>::VE;
  const unsigned bits = lane_hot ? group_bits(c, s, q, x, lead, len, n_groups) : 0u;
  if (__any_sync(kFull, (bits & (bits - 1u)) != 0u)) {
    warp_append_bits(c, s, bits, x, colbase + q * VE);
    return;
  }
  const unsigned mk = __ballot_sync(kFull, bits != 0u);
  if (!mk) return;
  if (s.n + __popc(mk) > kCapW) {
    warp_append_bits(c, s, bits, x, colbase + q * VE);  // compacts
    return;
  }
  if (bits) {
    const int i = __ffs(bits) - 1;
    const int pos = s.n + __popc(mk & lanemask_lt());
    float v = x[0];
#pragma unroll
    for (int k = 1; k < VE; ++k)
      if (i == k) v = x[k];
    s.x[pos] = v;
    s.col[pos] = colbase + q * VE + i;
  }
  s.n += __popc(mk);
}

// ---------------------------------------------------------------------------
// full tiles (every slot a column, first column 16-byte aligned): lane l holds
// 16-byte groups l, l + 32, ... in registers; one NaN-propagating max per lane
// decides whether any element needs a closer look
// ---------------------------------------------------------------------------
template <int DT>
constexpr int kGroupsPerLane = Ctx<DT>::TE / Ctx<DT>::VE / 32;

// Largest value of one 16-byte group in the filter domain (negated when NEG):
// NaN if any is NaN.  16-bit types reduce pairwise in their own format, which
// is exact (max is a selection).
template <int DT, bool NEG>
__device__ __forceinline__ float group_extreme(const uint4& v) {
  if constexpr (DT == NS_DTYPE_F32) {
    const float x0 = __uint_as_float(v.x), x1 = __uint_as_float(v.y);
    const float x2 = __uint_as_float(v.z), x3 = __uint_as_float(v.w);
    return NEG ? -fmin_nan(fmin_nan(x0, x1), fmin_nan(x2, x3)) : fmax_nan(fmax_nan(x0, x1), fmax_nan(x2, x3));
  } else {
    using P = typename std::conditional<DT == NS_DTYPE_BF16, __nv_bfloat162, __half2>::type;
    auto as2 = [](uint32_t u) {
      P p;
      memcpy(&p, &u, 4);
      return p;
    };
    auto op = [](P x, P y) { return NEG ? __hmin2_nan(x, y) : __hmax2_nan(x, y); };
    const P a = op(op(as2(v.x), as2(v.y)), op(as2(v.z), as2(v.w)));
    uint32_t u;
    memcpy(&u, &a, 4);
    const float lo = Elem<DT>::widen(uint16_t(u & 0xFFFFu)), hi = Elem<DT>::widen(uint16_t(u >> 16));
    return NEG ? -fmin_nan(lo, hi) : fmax_nan(lo, hi);
  }
}

template <int DT>
__device__ __forceinline__ void load_full(const uint8_t* st, uint4 (&v)[kGroupsPerLane<DT>]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kGroupsPerLane<DT>; ++k) v[k] = *reinterpret_cast<const uint4*>(st + (k * 32 + lane) * 16);
}

// FAST filter of a full tile: a per-lane mask of the groups whose max reaches
// tau (or is NaN) and one vote; hot groups are re-read from shared memory one
// per lane per round (lanes may work on different groups in one round).
template <int DT, bool NEG>
__device__ __forceinline__ unsigned full_hot_mask(const WarpCand& s, const uint8_t* st) {
  constexpr int G = kGroupsPerLane<DT>;
  unsigned gm = 0;
  uint4 v[G];
  load_full<DT>(st, v);
#pragma unroll
  for (int k = 0; k < G; ++k) gm |= (group_extreme<DT, NEG>(v[k]) < s.tau ? 0u : 1u) << k;
  return gm;
}

template <int DT, bool NEG>
__device__ __forceinline__ void fast_full(const Ctx<DT>& c, WarpCand& s, const uint8_t* st, int colbase,
                                          unsigned gm) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  const int lane = threadIdx.x & 31;
  while (__any_sync(kFull, gm != 0u)) {
    const bool h = gm != 0u;
    const int k = h ? __ffs(gm) - 1 : 0;
    gm &= gm - 1u;
    float x[VE];
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + (k * 32 + lane) * 16), x);
    bool cold = true;
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      if (NEG) x[i] = -x[i];
      cold = cold && (x[i] < s.tau);  // tau may have risen in this tile
    }
    const bool hh = h && !cold;
    if (__any_sync(kFull, hh)) group_append(c, s, k * 32 + lane, x, hh, 0, TE, TE / VE, colbase);
  }
}

// GREEDY of a full tile already in registers (gx: the groups' maxima).
template <int DT>
__device__ __forceinline__ void greedy_regs(const uint4 (&v)[kGroupsPerLane<DT>],
                                            const float (&gx)[kGroupsPerLane<DT>], int colbase, float& best,
                                            int& bidx) {
  constexpr int VE = Ctx<DT>::VE, G = kGroupsPerLane<DT>;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < G; ++k) {
    if (gx[k] <= best && bidx != INT_MAX) continue;
    float x[VE];
    unpack16<DT>(v[k], x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int col = colbase + (k * 32 + lane) * VE + i;
      if (better(x[i], col, best, bidx)) {
        best = x[i];
        bidx = col;
      }
    }
  }
}

// GREEDY of a full tile: per-lane running argmax under the full (value, first
// index, NaN first) order; groups whose max cannot win are skipped.
template <int DT>
__device__ __forceinline__ void greedy_full(const uint8_t* st, int colbase, float& best, int& bidx) {
  constexpr int VE = Ctx<DT>::VE, G = kGroupsPerLane<DT>;
  const int lane = threadIdx.x & 31;
  uint4 v[G];
  load_full<DT>(st, v);
#pragma unroll
  for (int k = 0; k < G; ++k) {
    if (group_extreme<DT, false>(v[k]) <= best && bidx != INT_MAX) continue;
    float x[VE];
    unpack16<DT>(v[k], x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int col = colbase + (k * 32 + lane) * VE + i;
      if (better(x[i], col, best, bidx)) {
        best = x[i];
        bidx = col;
      }
    }
  }
}

// FAST filter of one landed tile: two 16-byte groups per lane per step, each
// with its own vote; the common group is a shared load, a compare chain and
// a vote.
template <int DT, bool NEG>
__device__ __forceinline__ void fast_tile(const Ctx<DT>& c, WarpCand& s, int w, int t, const uint8_t* st, bool full) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  const int lane = threadIdx.x & 31;
  const int len = c.tile_len(w, t), lead = c.tile_lead(w, t);
  const int n_groups = (lead + len + VE - 1) / VE;
  const int colbase = w * c.pw + t * TE - lead;  // CTA-relative column of slot 0
  if (full) {
    fast_full<DT, NEG>(c, s, st, colbase, full_hot_mask<DT, NEG>(s, st));
    return;
  }
  for (int q0 = 0; q0 < n_groups; q0 += 64) {
    const int qa = q0 + lane, qb = q0 + 32 + lane;
    float xa[VE], xb[VE];
    load_group<DT, NEG>(st, qa, n_groups, xa);
    load_group<DT, NEG>(st, qb, n_groups, xb);
    bool ca = true, cb = true;
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      ca = ca && (xa[i] < s.tau);
      cb = cb && (xb[i] < s.tau);
    }
    if (__any_sync(kFull, !ca)) group_append(c, s, qa, xa, !ca, lead, len, n_groups, colbase);
    if (__any_sync(kFull, !cb)) group_append(c, s, qb, xb, !cb, lead, len, n_groups, colbase);
  }
}

// FAST handling of one penalised history value (all lanes, one per lane).
template <int DT>
__device__ __forceinline__ void fast_emit(const Ctx<DT>& c, WarpCand& s, bool has, float xp, int col) {
  const bool bad = has && (xp != xp || xp == INFINITY);
  if (bad) atomicOr(&c.m->flags, F_NAN);
  const float v[1] = {xp};
  warp_append_bits(c, s, (has && !bad && xp >= s.tau && xp > -INFINITY) ? 1u : 0u, v, col);
}

// GREEDY of one landed tile: per-lane running argmax under the full (value,
// first index, NaN first) order; the penalised history values arrive out of
// column order.  A group whose NaN-propagating max cannot win is skipped.
template <int DT>
__device__ __forceinline__ void greedy_group(const float (&x)[Ctx<DT>::VE], int q, int lead, int len, int n_groups,
                                             int colbase, float& best, int& bidx) {
  constexpr int VE = Ctx<DT>::VE;
  float m = x[0];
#pragma unroll
  for (int i = 1; i < VE; ++i) m = fmax_nan(m, x[i]);
  if (m <= best && bidx != INT_MAX) return;
#pragma unroll
  for (int i = 0; i < VE; ++i) {
    const int e = q * VE + i;
    const bool valid = (q < n_groups) && e >= lead && e < lead + len;
    if (valid && better(x[i], colbase + e, best, bidx)) {
      best = x[i];
      bidx = colbase + e;
    }
  }
}

template <int DT>
__device__ __forceinline__ void greedy_tile(const Ctx<DT>& c, int w, int t, const uint8_t* st, float& best,
                                            int& bidx, bool full) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  const int lane = threadIdx.x & 31;
  const int len = c.tile_len(w, t), lead = c.tile_lead(w, t);
  const int n_groups = (lead + len + VE - 1) / VE;
  const int colbase = c.c0 + w * c.pw + t * TE - lead;  // call-local column of slot 0
  if (full) {
    greedy_full<DT>(st, colbase, best, bidx);
    return;
  }
  for (int q0 = 0; q0 < n_groups; q0 += 64) {
    const int qa = q0 + lane, qb = q0 + 32 + lane;
    float xa[VE], xb[VE];
    load_group<DT, false>(st, qa, n_groups, xa);
    load_group<DT, false>(st, qb, n_groups, xb);
    greedy_group<DT>(xa, qa, lead, len, n_groups, colbase, best, bidx);
    greedy_group<DT>(xb, qb, lead, len, n_groups, colbase, best, bidx);
  }
}

// Leading tiles of warp w that are full and start on a 16-byte boundary (the
// register paths and single-copy issue); the alignment is the same for every
// tile of the warp because a tile is a multiple of 16 bytes.
template <int DT>
__device__ __forceinline__ int full_tiles(const Ctx<DT>& c, int w) {
  if (c.w1(w) <= c.w0(w) || c.tile_head(w, 0) != 0) return 0;
  return (c.w1(w) - c.w0(w)) / Ctx<DT>::TE;
}

// Largest finite value of the lane's slots of a landed tile in the filter
// domain (-inf if none; a lane holding a NaN or +inf contributes nothing).
template <int DT, bool NEG>
__device__ __forceinline__ float tile_lane_max(const Ctx<DT>& c, int w, int t, const uint8_t* st) {
  constexpr int VE = Ctx<DT>::VE;
  const int lane = threadIdx.x & 31;
  const int len = c.tile_len(w, t), lead = c.tile_lead(w, t);
  if (t < full_tiles(c, w)) {
    uint4 v[kGroupsPerLane<DT>];
    load_full<DT>(st, v);
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kGroupsPerLane<DT>; ++k) {
      const float g = group_extreme<DT, NEG>(v[k]);
      if (g > -INFINITY && g < INFINITY) m = fmaxf(m, g);  // a group holding NaN or +inf is left out
    }
    return m;
  }
  const int n_groups = (lead + len + VE - 1) / VE;
  float tmax = -INFINITY;
  for (int q = lane; q < n_groups; q += 32) {
    float x[VE];
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int e = q * VE + i;
      const float xk = NEG ? -x[i] : x[i];
      if (e >= lead && e < lead + len && xk > -INFINITY && xk < INFINITY) tmax = fmaxf(tmax, xk);
    }
  }
  return tmax;
}

// ---------------------------------------------------------------------------
// SOFTMAX rows (top-k and top-p both off): one pass.  Per warp tile, the
// largest scaled value ym = rn(xmax / |T|) and D = sum of expf(rn(x / |T|) - ym)
// over its finite values, in float64; the draw is located afterwards from the
// tiles' masses scaled by expf(ym - M) and one tile is read again.
// ---------------------------------------------------------------------------
__device__ __forceinline__ double* softmax_tile_mass(void* tacc) { return reinterpret_cast<double*>(tacc); }
template <int DT>
__device__ __forceinline__ float* softmax_tile_max(const Ctx<DT>& c) {
  return reinterpret_cast<float*>(softmax_tile_mass(c.tacc) + kWarps * c.tpw);
}

// x / T within one ulp from r = rn(1 / T): the product's remainder, exact by
// FMA, corrects the quotient once (Newton-Raphson; Markstein, IBM J. Res.
// Dev. 34(1), 1990).  A quotient that overflows comes out NaN or infinite.
__device__ __forceinline__ float quot_nr(float x, float T, float r) {
  const float q = x * r;
  return fmaf(fmaf(-q, T, x), r, q);
}

// exp(d) for d <= ~0 as 2^(d log2 e), the product kept as hi + lo: log2 e is
// split into two fp32 parts (Cody and Waite's two-constant reduction), hi =
// rn(d L1), lo = the product's rounding error (FMA) plus d L2.  2^hi by the
// hardware approximation, the lo term to first order: relative error ~2^-22.
__device__ __forceinline__ float exp_split(float d) {
  constexpr float L1 = 1.4426950216293335f;       // fp32 nearest to log2(e)
  constexpr float L2 = 1.925963033500011e-08f;    // log2(e) - L1
  constexpr float LN2 = 0.693147182464599609375f;
  const float hi = d * L1;
  const float lo = fmaf(d, L2, fmaf(d, L1, -hi));
  const float p = ex2_approx(hi);
  return fmaf(p * lo, LN2, p);
}

// Softmax weight of a value x (filter domain) in a tile whose largest scaled
// value is ym: exp(x / |T| - ym).  A quotient that overflows (NaN or -inf)
// clamps to weight 0; a tile whose own maximum overflows reports the row
// instead, so no value above ym can overflow.
__device__ __forceinline__ float softmax_weight(float x, float ym, float T, float r) {
  return exp_split(fmaxf(quot_nr(x, T, r) - ym, -1000.0f));
}

// SOFTMAX per-tile mass.  FULL: every slot is a column and slot 0 is column 0.
template <int DT, bool NEG, bool FULL>
__device__ __forceinline__ void mass_tile_t(const Ctx<DT>& c, int w, int t, const uint8_t* st) {
  constexpr int VE = Ctx<DT>::VE;
  const int lane = threadIdx.x & 31;
  const int len = FULL ? Ctx<DT>::TE : c.tile_len(w, t), lead = FULL ? 0 : c.tile_lead(w, t);
  const int n_groups = (lead + len + VE - 1) / VE;
  float mx = -INFINITY;  // NaN-propagating: NaN or +inf anywhere shows here
  for (int q = lane; q < n_groups; q += 32) {
    const uint4 v = *reinterpret_cast<const uint4*>(st + q * 16);
    if (FULL) {
      mx = fmax_nan(mx, group_extreme<DT, NEG>(v));
    } else {
      float x[VE];
      unpack16<DT>(v, x);
#pragma unroll
      for (int i = 0; i < VE; ++i)
        if (q * VE + i >= lead && q * VE + i < lead + len) mx = fmax_nan(mx, NEG ? -x[i] : x[i]);
    }
  }
  float ym = -INFINITY;
  double acc = 0.0;
  if (__any_sync(kFull, !(mx < INFINITY))) {
    if (lane == 0) atomicOr(&c.m->flags, F_NAN);
  } else {
    const float xm = key2f(__reduce_max_sync(kFull, f2key(mx)));
    if (xm > -INFINITY) {
      ym = __fdiv_rn(xm, c.Tabs);
      if (!(ym < INFINITY)) {  // x / T overflows: the reference's softmax is NaN
        if (lane == 0) atomicOr(&c.m->flags, F_NAN);
        ym = -INFINITY;
      } else {
        // a 16-byte group's weights summed pairwise in fp32, then in float64
        const float rT = __frcp_rn(c.Tabs);
        for (int q = lane; q < n_groups; q += 32) {
          float x[VE];
          unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
          float wv[VE];
#pragma unroll
          for (int i = 0; i < VE; ++i) {
            const bool in = FULL || (q * VE + i >= lead && q * VE + i < lead + len);
            wv[i] = in ? softmax_weight(NEG ? -x[i] : x[i], ym, c.Tabs, rT) : 0.0f;
          }
#pragma unroll
          for (int h = VE / 2; h >= 1; h >>= 1)
#pragma unroll
            for (int i = 0; i < h; ++i) wv[i] += wv[i + h];
          acc += double(wv[0]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
      }
    }
  }
  if (lane == 0) {
    softmax_tile_mass(c.tacc)[w * c.tpw + t] = acc;
    softmax_tile_max(c)[w * c.tpw + t] = ym;
  }
}

template <int DT, bool NEG>
__device__ __forceinline__ void mass_tile(const Ctx<DT>& c, int w, int t, const uint8_t* st, bool full) {
  if (full)
    mass_tile_t<DT, NEG, true>(c, w, t, st);
  else
    mass_tile_t<DT, NEG, false>(c, w, t, st);
}

// ---------------------------------------------------------------------------
// FAST threshold sharing without block barriers.  A warp publishes a bound
// from v_w, the kq-th largest (kq = ceil(K / kWarps)) element it holds; every
// element of the warp's columns >= its own tau is held, so v_w has kq elements
// of the CTA at or above it.  Once all kWarps warps have published, the CTA has
// at least kWarps * kq >= K elements >= min_w v_w: a lower bound of its K-th
// largest.  The published value is already a filter bound b_w <=
// scaled_lower_bound(v_w) (fast_lower_bound), so the minimum of the published
// bounds is at most the bound of the smallest v_w, which is a valid filter for
// the CTA.  Published values only grow, so a stale read is still valid.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int share_kq(int K) { return (K + kWarps - 1) / kWarps; }

// kq-th largest (with multiplicity) of one key per lane; 0 if fewer than kq
// non-zero keys.
__device__ __forceinline__ uint32_t warp_kth_lanes(uint32_t key, int kq) {
  const int lane = threadIdx.x & 31;
  uint32_t res = 0;
  for (int j = 0; j < kq; ++j) {
    res = __reduce_max_sync(kFull, key);
    if (res == 0u) break;
    const unsigned b = __ballot_sync(kFull, key == res);
    if (lane == __ffs(b) - 1) key = 0u;
  }
  return res;
}

// Raise tau to the shared bound (all lanes call).
template <int DT>
__device__ __forceinline__ void read_shared_tau(const Ctx<DT>& c, WarpCand& s) {
  const int lane = threadIdx.x & 31;
  const uint32_t p = (lane < kWarps) ? static_cast<volatile uint32_t*>(c.m->pub)[lane] : 0xFFFFFFFFu;
  const uint32_t mn = __reduce_min_sync(kFull, p);
  if (mn != 0u) s.tau = fmaxf(s.tau, key2f(mn));
}

// Publish this warp's bound from the kq-th largest value v (key; 0 = none).
template <int DT>
__device__ __forceinline__ void publish_key(const Ctx<DT>& c, uint32_t v) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0 && v != 0u) {
    const uint32_t b = f2key(fast_lower_bound(key2f(v), c.Tabs));
    volatile uint32_t* pub = c.m->pub;
    if (b > pub[warp]) pub[warp] = b;
  }
  __syncwarp();
}

// The kq-th largest of the per-lane maxima of the buffer: kq distinct held
// elements are at or above it.
template <int DT>
__device__ __forceinline__ void publish_bound(const Ctx<DT>& c, const WarpCand& s) {
  if (s.ovf) return;
  const int lane = threadIdx.x & 31;
  uint32_t lm = 0;
#pragma unroll
  for (int q = 0; q < kPerLane; ++q) {
    const int i = q * 32 + lane;
    if (i < s.n) lm = max(lm, f2key(s.x[i]));
  }
  publish_key(c, warp_kth_lanes(lm, share_kq(c.K)));
}

// Stream this warp's tiles from t_begin (its first kWStages copies were issued
// before the history prologue; tiles below n_ready were already waited for and
// masked).  mode: GREEDY or FAST.  Returns false if a bounded wait gave up
// (F_TIMEOUT is set); in-flight copies are drained first.
// One instantiation per (mode, sign of T) keeps each loop's code compact.
template <int DT, int MODE, bool NEG>
__device__ __forceinline__ bool stream_warp_t(const Ctx<DT>& c, uint64_t policy, int t_begin, int n_ready,
                                              WarpCand& s, float& best, int& bidx) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = c.wtiles(w);
  const int nfull = full_tiles(c, w);
  for (int t = t_begin; t < nt; ++t) {
    const int sidx = t % kWStages;
    uint8_t* st = c.stage(w, sidx);
    if (t >= n_ready) {
      const bool ok = mbar_wait_bounded(c.sbar(w, sidx), uint32_t(t / kWStages) & 1u);
      if (!__all_sync(kFull, ok)) {
        if (lane == 0) {
          atomicOr(&c.m->flags, F_TIMEOUT);
          for (int u = t; u < min(nt, t + kWStages); ++u)
            mbar_wait_bounded(c.sbar(w, u % kWStages), uint32_t(u / kWStages) & 1u);
        }
        __syncwarp();
        return false;
      }
      if (c.pen) {
        mask_tile(c, w, t, st);
        __syncwarp();
      }
    }
    // Full tiles: the stage is refilled as soon as its bytes are no longer
    // needed -- GREEDY once the tile is in registers, FAST once no group of
    // it reaches tau (every load has been waited for by then).
    auto issue_next = [&]() {
      if (lane == 0 && t + kWStages < nt) {
        const int tn = t + kWStages;
        if (tn < nfull)
          issue_full_tile(c, w, tn, tn % kWStages, policy);
        else
          issue_tile(c, w, tn, tn % kWStages, policy);
      }
    };
    if constexpr (MODE == MODE_GREEDY) {
      if (t < nfull) {
        constexpr int G = kGroupsPerLane<DT>;
        uint4 v[G];
        float gx[G];
        load_full<DT>(st, v);
#pragma unroll
        for (int k = 0; k < G; ++k) gx[k] = group_extreme<DT, false>(v[k]);
        __syncwarp();
        issue_next();
        greedy_regs<DT>(v, gx, c.c0 + w * c.pw + t * Ctx<DT>::TE, best, bidx);  // full tiles: lead 0
        continue;
      }
    }
    if constexpr (MODE == MODE_FAST) {
      if (t < nfull && !s.ovf) {
        const unsigned gm = full_hot_mask<DT, NEG>(s, st);
        const bool hot = __any_sync(kFull, gm != 0u);
        if (!hot) issue_next();
        else fast_full<DT, NEG>(c, s, st, w * c.pw + t * Ctx<DT>::TE, gm);
        if (t == 1 || t == 4 || t == 9) publish_bound(c, s);
        read_shared_tau(c, s);
        if (hot) {
          __syncwarp();
          issue_next();
        }
        continue;
      }
    }
    if constexpr (MODE == MODE_GREEDY) {
      greedy_tile(c, w, t, st, best, bidx, t < nfull);
    } else if constexpr (MODE == MODE_SOFTMAX) {
      mass_tile<DT, NEG>(c, w, t, st, t < nfull);
    } else {
      if (!s.ovf) fast_tile<DT, NEG>(c, s, w, t, st, t < nfull);
      if constexpr (MODE == MODE_NUCLEUS) mass_tile<DT, NEG>(c, w, t, st, t < nfull);  // even after an overflow
      if (!s.ovf) {
        if (t == 1 || t == 4 || t == 9) publish_bound(c, s);
        read_shared_tau(c, s);
      }
    }
    __syncwarp();
    if (lane == 0 && t + kWStages < nt) {
      const int tn = t + kWStages;
      if (tn < nfull)
        issue_full_tile(c, w, tn, tn % kWStages, policy);
      else
        issue_tile(c, w, tn, tn % kWStages, policy);
    }
  }
  return true;
}

template <int DT>
__device__ __forceinline__ bool stream_warp(const Ctx<DT>& c, int mode, uint64_t policy, int t_begin, int n_ready,
                                            WarpCand& s, float& best, int& bidx) {
  switch (mode) {
    case MODE_GREEDY: return stream_warp_t<DT, MODE_GREEDY, false>(c, policy, t_begin, n_ready, s, best, bidx);
    case MODE_SOFTMAX:
      return c.neg ? stream_warp_t<DT, MODE_SOFTMAX, true>(c, policy, t_begin, n_ready, s, best, bidx)
                   : stream_warp_t<DT, MODE_SOFTMAX, false>(c, policy, t_begin, n_ready, s, best, bidx);
    case MODE_NUCLEUS:
      return c.neg ? stream_warp_t<DT, MODE_NUCLEUS, true>(c, policy, t_begin, n_ready, s, best, bidx)
                   : stream_warp_t<DT, MODE_NUCLEUS, false>(c, policy, t_begin, n_ready, s, best, bidx);
    default:
      return c.neg ? stream_warp_t<DT, MODE_FAST, true>(c, policy, t_begin, n_ready, s, best, bidx)
                   : stream_warp_t<DT, MODE_FAST, false>(c, policy, t_begin, n_ready, s, best, bidx);
  }
}

// ---------------------------------------------------------------------------
// block-level helpers for the cluster leader
// ---------------------------------------------------------------------------
// K-th largest (1-based) of the values visited by `for_each` (called by every
// thread with a per-thread share).  False if fewer than K values were visited.
// 8-bit MSB-first radix select with shared-memory histograms.
template <class ForEach>
__device__ bool block_radix_kth(Misc* m, int K, ForEach for_each, uint32_t* out_key) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  int krem = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < kBins; i += kThreads) m->hist[i] = 0;
    __syncthreads();
    for_each([&](float x) {
      const uint32_t k = f2key(x);
      if ((k & pmask) == prefix) atomicAdd(&m->hist[(k >> shift) & 0xFFu], 1u);
    });
    __syncthreads();
    if (warp == 0) {
      uint32_t cnt[8];
      uint32_t local = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cnt[q] = m->hist[255 - 8 * lane - q];
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
        if (lane == 0) m->r_digit = -1;
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
        m->r_digit = d;
        m->r_krem = kr;
      }
    }
    __syncthreads();
    const int d = m->r_digit;
    if (d < 0) return false;
    prefix |= uint32_t(d) << shift;
    pmask |= 0xFFu << shift;
    krem = m->r_krem;
    __syncthreads();
  }
  *out_key = prefix;
  return true;
}

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

// Orders n distinct keys by before(a, b) into out[]: counted into kBins
// buckets (shared atomics), placed by bucket into tmp[], then ranked inside
// their bucket.  bucket(k) in [0, kBins) must follow the order: bucket(a) <
// bucket(b) implies before(a, b).  O(n) plus the squares of the bucket sizes.
// Uses Misc::hist and Misc::i_red; all threads of the block; a barrier follows.
template <class Bucket, class Before>
__device__ void bucket_sort(Misc* m, const uint64_t* in, int n, uint64_t* tmp, uint64_t* out, Bucket bucket,
                            Before before) {
  static_assert(kBins == kThreads, "one bucket per thread in the scan");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* cnt = m->hist;
  cnt[tid] = 0u;
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) atomicAdd(&cnt[bucket(in[i])], 1u);
  __syncthreads();
  const int v = int(cnt[tid]);
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) m->i_red[warp] = incl;
  __syncthreads();
  int base = 0;
  for (int w = 0; w < warp; ++w) base += m->i_red[w];
  cnt[tid] = uint32_t(base + incl - v);  // first slot of bucket tid
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    const uint64_t k = in[i];
    tmp[atomicAdd(&cnt[bucket(k)], 1u)] = k;
  }
  __syncthreads();  // cnt[b]: one past the last slot of bucket b
  for (int p = tid; p < n; p += kThreads) {
    const uint64_t k = tmp[p];
    const int b = bucket(k);
    const int s0 = b ? int(cnt[b - 1]) : 0, s1 = int(cnt[b]);
    int r = 0;
    for (int q = s0; q < s1; ++q) r += before(tmp[q], k) ? 1 : 0;
    out[s0 + r] = k;
  }
  __syncthreads();
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

constexpr int kSmallN = 128;
constexpr int kSmallRank = 2048;  // finalise: kept sets up to this size are bucket-sorted by id
static_assert(2 * kSmallRank <= kMergeCap, "the id keys and their bucket staging fit the finalise keys area");

template <int DT>
__device__ void finalize_small_sorted(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, int n,
                                      double norm = -1.0);

// Leader, FAST rows with n <= kSmallN survivors: sort by rank counting (thread
// i owns survivor i), then one warp computes the softmax prefix sums with
// shuffles (4 positions per lane).
template <int DT>
__device__ void finalize_small(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, int n) {
  const int tid = threadIdx.x;
  const float* my = reinterpret_cast<const float*>(c.stages);
  const int* mid = reinterpret_cast<const int*>(c.stages + size_t(a.merge_cap) * 4);
  float* sy = reinterpret_cast<float*>(c.stages + size_t(a.merge_cap) * 8);
  int* sid = reinterpret_cast<int*>(sy + kSmallN);
  if (tid < n) {  // position in (y desc, id asc) order
    const float yi = my[tid] + 0.0f;
    const int ii = mid[tid];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const float yj = my[j] + 0.0f;
      rank += (yj > yi || (yj == yi && mid[j] < ii)) ? 1 : 0;
    }
    sy[rank] = yi;
    sid[rank] = ii;
  }
  __syncthreads();
  finalize_small_sorted(c, a, row, topp, n);
}

// Leader, FAST rows: n <= kSmallN survivors already in (y desc, id asc) order
// in sy[] / sid[]; one warp computes the softmax prefix sums with shuffles (4
// positions per lane).
// norm > 0: the softmax's normaliser is the row's total mass (top-k off), not
// the survivors' sum.
template <int DT>
__device__ void finalize_small_sorted(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, int n,
                                      double norm) {
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* sy = reinterpret_cast<float*>(c.stages + size_t(a.merge_cap) * 8);
  int* sid = reinterpret_cast<int*>(sy + kSmallN);
  float* se = reinterpret_cast<float*>(sid + kSmallN);
  int* kid = reinterpret_cast<int*>(se + kSmallN);
  float* kw = reinterpret_cast<float*>(kid + kSmallN);
  const float M = sy[0];
  if (!(M < INFINITY)) {
    if (tid == 0) a.out_ids[row] = NS_ERR_INVALID_DISTRIBUTION;
    return;
  }
  if (warp == 0) {
    // softmax weights and the top-p cut: sorted position j+1 survives iff
    // cumsum[j] <= p (reference sampler.py:127-131)
    double e[4], local = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = lane * 4 + k;
      const float w = (j < n) ? expf(__fsub_rn(sy[j], M)) : 0.0f;
      if (j < n) se[j] = w;
      e[k] = double(w);
      local += e[k];
    }
    double incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    const double total = __shfl_sync(kFull, incl, 31);
    int L = n;
    if (topp > 0.0f && topp < 1.0f) {
      int cnt = 0;
      double run = incl - local;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int j = lane * 4 + k;
        run += e[k];
        cnt += (j <= n - 2 && run <= double(topp) * (norm > 0.0 ? norm : total)) ? 1 : 0;
      }
      L = 1 + int(__reduce_add_sync(kFull, unsigned(cnt)));
    }
    if (lane == 0) m->r_krem = L;
  }
  __syncthreads();
  const int L = m->r_krem;
  if (tid < L) {  // ascending-id order among the kept positions
    const int ii = sid[tid];
    int r2 = 0;
    for (int j = 0; j < L; ++j) r2 += (sid[j] < ii) ? 1 : 0;
    kid[r2] = ii;
    kw[r2] = se[tid];
  }
  __syncthreads();
  if (warp == 0) {
    // inverse CDF: the first kept id whose running weight exceeds u * total
    const float u = a.uniforms ? c.u_pre : philox_uniform(a.seed, a.offset, uint64_t(row));
    double e[4], local = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = lane * 4 + k;
      e[k] = (j < L) ? double(kw[j]) : 0.0;
      local += e[k];
    }
    double incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    const double total = __shfl_sync(kFull, incl, 31);
    const double target = double(u) * total;
    int first = INT_MAX;
    double run = incl - local;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = lane * 4 + k;
      run += e[k];
      if (first == INT_MAX && j < L && run > target) first = j;
    }
    first = int(__reduce_min_sync(kFull, unsigned(first)));
    if (lane == 0) a.out_ids[row] = int64_t(kid[first == INT_MAX ? L - 1 : first]) + a.vocab_offset;
  }
}

// Leader, FAST rows: survivors sorted by (y desc, id asc); softmax; top-p cut
// (keep sorted j iff j == 0 or cumsum[j-1] <= p, reference sampler.py:122-131);
// then the inverse-CDF draw over the kept ids in ascending id order.
// presorted: my[] / mid[] already hold that order.  norm > 0: the softmax's
// normaliser is the row's total mass (top-k off), not the survivors' sum.
template <int DT>
__device__ void finalize_row(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, double norm = -1.0,
                             bool presorted = false) {
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
  if (n <= kSmallN && !presorted) {
    finalize_small(c, a, row, topp, n);
    return;
  }
  if (!presorted) {
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
  }
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
        [&](int i, double incl, double total) {
          cnt += (i <= n - 2 && incl <= p * (norm > 0.0 ? norm : total)) ? 1 : 0;
        });
    L = 1 + block_sum_int(m, cnt);
  }
  const uint64_t* ord = keys;  // (id << 32 | weight) in ascending id order
  if (L <= kSmallRank) {  // bucket sort by id range (ids are distinct)
    for (int i = tid; i < L; i += kThreads)
      keys[i] = (uint64_t(uint32_t(mid[i])) << 32) | uint64_t(__float_as_uint(my[i]));
    __syncthreads();
    int sh = 0;  // ids < vocab_total <= 2^(8 + sh)
    while ((a.vocab_total - 1) >> (8 + sh)) ++sh;
    uint64_t* tmp = keys + kSmallRank;
    uint64_t* out = reinterpret_cast<uint64_t*>(my);  // my[] and mid[] are dead
    bucket_sort(
        m, keys, L, tmp, out, [&](uint64_t k) { return int(uint32_t(k >> 32) >> sh); },
        [](uint64_t x, uint64_t y) { return x < y; });
    ord = out;
  } else {
    int n3 = 1;
    while (n3 < L) n3 <<= 1;
    for (int i = tid; i < n3; i += kThreads)
      keys[i] = (i < L) ? ((uint64_t(uint32_t(mid[i])) << 32) | uint64_t(__float_as_uint(my[i]))) : ~0ull;
    __syncthreads();
    bitonic_sort_u64(keys, n3, false);
  }
  const float u = a.uniforms ? c.u_pre : philox_uniform(a.seed, a.offset, uint64_t(row));
  if (tid == 0) m->choose = INT_MAX;
  __syncthreads();
  int first = INT_MAX;
  block_chunk_scan(
      m, L, [&](int i) { return double(__uint_as_float(uint32_t(ord[i]))); },
      [&](int i, double incl, double total) {
        if (first == INT_MAX && incl > double(u) * total) first = i;
      });
  if (first != INT_MAX) atomicMin(&m->choose, first);
  __syncthreads();
  if (tid == 0) {
    const int ch = (m->choose == INT_MAX) ? L - 1 : m->choose;
    a.out_ids[row] = int64_t(uint32_t(ord[ch] >> 32)) + a.vocab_offset;
  }
}

// K-th largest (1-based) of the non-zero keys held in registers by all
// threads of the block (zero = empty slot).  8-bit MSB-first radix select
// with one shared-memory histogram per round (12 block barriers).  Returns
// false if fewer than K keys are present.
template <int R>
__device__ __forceinline__ bool block_kth_regs(Misc* m, const uint32_t (&key)[R], int K, uint32_t* out_key) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, pmask = 0;
  int krem = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    m->hist[tid] = 0;  // kBins == kThreads
    __syncthreads();
#pragma unroll
    for (int q = 0; q < R; ++q)
      if (key[q] != 0u && (key[q] & pmask) == prefix) atomicAdd(&m->hist[(key[q] >> shift) & 0xFFu], 1u);
    __syncthreads();
    if (warp == 0) {
      uint32_t cnt[8];
      uint32_t local = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cnt[q] = m->hist[255 - 8 * lane - q];
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
        if (lane == 0) m->r_digit = -1;
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
        m->r_digit = d;
        m->r_krem = kr;
      }
    }
    __syncthreads();
    const int d = m->r_digit;
    if (d < 0) return false;
    prefix |= uint32_t(d) << shift;
    pmask |= 0xFFu << shift;
    krem = m->r_krem;
  }
  *out_key = prefix;
  return true;
}

// Leader, FAST rows whose union of survivors has at most kRankMax entries:
// every survivor becomes the key (f2key(y) << 32) | ~id, y = rn(x / |T|), so
// keys order by (y desc, id asc) and are distinct.  gather_keys copies the
// union (read through distributed shared memory) before the cluster's last
// barrier; rank_finalize sorts it by counting, for each key, the keys above
// it, and takes the top-k with its ties at the k-th scaled value.
constexpr int kRankMax = 1024;
static_assert(kRankMax * 8 <= kCandBytes, "sorted keys of a single-CTA row fit the candidate buffers");
static_assert((kCapW + 1) * 8 <= kWStageStride, "a warp's keys (padded) fit its first stage");
// keys[kRankMax] and sorted[kRankMax] in the stage area, past the merge lists
// (y, id: kMergeCap * 8 bytes), finalize_small's arrays (5 * kSmallN * 4) and
// finalize_row's sort keys for up to kRankMax survivors
constexpr size_t kRankKeysOff = size_t(kMergeCap) * 8 + size_t(kRankMax) * 8;
static_assert(size_t(kMergeCap) * 8 + 5 * kSmallN * 4 <= size_t(kMergeCap) * 8 + size_t(kRankMax) * 8,
              "finalize_small's arrays fit below the rank keys");
static_assert(kRankKeysOff + 2 * size_t(kRankMax) * 8 <= size_t(kStageBytes), "rank-sort keys fit the stage area");
constexpr int kMergeStage = kMergeCap;  // union keys the merge stages (32 KB at the stage area's start)
static_assert(size_t(kMergeStage) * 8 <= kRankKeysOff, "staged lists end before the sorted keys");

template <int DT>
__device__ __forceinline__ void gather_keys(const Ctx<DT>& c, cg::cluster_group& cluster, int CL) {
  Misc* m = c.m;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t* keys = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff);
  const int nl = CL * kWarps;
  for (int l = warp; l < nl; l += kWarps) {
    const int r = l / kWarps, wl = l % kWarps;
    const int o = m->roff[l], nlst = m->roff[l + 1] - o;
    const float* rcx = cluster.map_shared_rank(c.cx, r) + wl * kCapW;
    const int* rcid = cluster.map_shared_rank(c.cid, r) + wl * kCapW;
    const int c0r = m->rc0[r];
    for (int i = lane; i < nlst; i += 32) {
      const float y = __fdiv_rn(rcx[i], c.Tabs) + 0.0f;  // -0 and +0 tie
      keys[o + i] = (uint64_t(f2key(y)) << 32) | uint64_t(~uint32_t(rcid[i] + c0r));
    }
  }
  if (threadIdx.x == 0 && (m->roff[nl] & 1)) keys[m->roff[nl]] = 0ull;  // pad to whole pairs
}

template <int DT>
__device__ void finalize_keys(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, const uint64_t* sorted,
                              int n, int n_all, double norm = -1.0);

template <int DT>
__device__ void rank_finalize(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, int n) {
  const int tid = threadIdx.x;
  const uint64_t* keys = reinterpret_cast<const uint64_t*>(c.stages + kRankKeysOff);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff) + kRankMax;
  if (n == 0) {  // nothing finite (a vocab-parallel slice may legitimately hold none)
    if (tid == 0) a.out_ids[row] = a.vp_keys ? 0 : NS_ERR_INVALID_DISTRIBUTION;
    return;
  }
  for (int i = tid; i < n; i += kThreads) {
    const uint64_t ki = keys[i];
    int r0 = 0, r1 = 0;
#pragma unroll 4
    for (int j = 0; j < n; j += 2) {
      const ulonglong2 p = *reinterpret_cast<const ulonglong2*>(keys + j);
      r0 += (p.x > ki) ? 1 : 0;
      r1 += (p.y > ki) ? 1 : 0;
    }
    sorted[r0 + r1] = ki;
  }
  __syncthreads();
  finalize_keys(c, a, row, topp, sorted, n, n);
}

// The first n keys of the sorted union (descending) are in sorted[] (outside
// the first 32 KB + 2.5 KB of the stage area, which the finalise reuses); n_all >=
// n survivors exist in total.  Top-k keeps every key whose scaled value ties
// the k-th (reference sampler.py:116-121); each warp finds the end of the tie
// run itself.  A tie run that reaches past the n placed keys overflows.
template <int DT>
__device__ void finalize_keys(const Ctx<DT>& c, const KArgs& a, int64_t row, float topp, const uint64_t* sorted,
                              int n, int n_all, double norm) {
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31;
  if (n == 0) {  // nothing finite (a vocab-parallel slice may legitimately hold none)
    if (tid == 0) a.out_ids[row] = a.vp_keys ? 0 : NS_ERR_INVALID_DISTRIBUTION;
    return;
  }
  const int kk = min(c.K, n);
  const uint32_t yk = uint32_t(sorted[kk - 1] >> 32);
  int nfin = n;
  for (int j0 = kk; j0 < n; j0 += 32) {
    const int j = j0 + lane;
    const unsigned b = __ballot_sync(kFull, j < n && uint32_t(sorted[j] >> 32) < yk);
    if (b) {
      nfin = j0 + __ffs(b) - 1;
      break;
    }
  }
  if (nfin == n && n_all > n) {
    if (tid == 0) a.out_ids[row] = NS_ERR_CANDIDATE_OVERFLOW;
    return;
  }
  if (a.vp_keys) {  // vocab-parallel local step: the survivors are the record
    if (nfin > a.vp_cap) {
      if (tid == 0) a.out_ids[row] = NS_ERR_CANDIDATE_OVERFLOW;
      return;
    }
    int64_t* rk = a.vp_keys + row * a.vp_cap;
    for (int i = tid; i < nfin; i += kThreads) {
      const uint32_t gid = ~uint32_t(sorted[i]) + uint32_t(a.vocab_offset);
      rk[i] = int64_t((sorted[i] & 0xFFFFFFFF00000000ull) | uint64_t(~gid));
    }
    if (tid == 0) a.out_ids[row] = nfin;
    return;
  }
  if (nfin <= kSmallN) {
    float* sy = reinterpret_cast<float*>(c.stages + size_t(a.merge_cap) * 8);
    int* sid = reinterpret_cast<int*>(sy + kSmallN);
    if (tid < nfin) {
      sy[tid] = key2f(uint32_t(sorted[tid] >> 32));
      sid[tid] = int(~uint32_t(sorted[tid]));
    }
    __syncthreads();
    finalize_small_sorted(c, a, row, topp, nfin, norm);
    return;
  }
  float* my = reinterpret_cast<float*>(c.stages);
  int* mid = reinterpret_cast<int*>(c.stages + size_t(a.merge_cap) * 4);
  for (int i = tid; i < nfin; i += kThreads) {
    my[i] = key2f(uint32_t(sorted[i] >> 32));
    mid[i] = int(~uint32_t(sorted[i]));
  }
  if (tid == 0) m->n_merge = nfin;
  __syncthreads();
  finalize_row(c, a, row, topp, norm, true);
}

// Merge nl descending lists of distinct keys (list l at lists[roff[l] ..
// roff[l + 1])) into sorted[0 .. min(n, kRankMax)): a key's position is its
// index in its own list plus, for every other list, the keys above it (binary
// search).  All threads of the block call it; a barrier follows.
__device__ __forceinline__ void place_sorted_lists(const uint64_t* lists, const int* roff, int nl, int n,
                                                   uint64_t* sorted) {
  for (int e = threadIdx.x; e < n; e += kThreads) {
    int r = 0;
    while (roff[r + 1] <= e) ++r;
    const uint64_t key = lists[e];
    int pos = e - roff[r];
    for (int r2 = 0; r2 < nl; ++r2) {
      if (r2 == r) continue;
      const uint64_t* l2 = lists + roff[r2];
      int lo = 0, hi = roff[r2 + 1] - roff[r2];
      while (lo < hi) {  // keys of list r2 above `key`
        const int mid = (lo + hi) >> 1;
        if (l2[mid] > key)
          lo = mid + 1;
        else
          hi = mid;
      }
      pos += lo;
    }
    if (pos < kRankMax) sorted[pos] = key;
  }
  __syncthreads();
}

// Number of keys kept by top-k with ties: the first k of the descending keys
// and every later key whose scaled value ties the k-th (reference
// sampler.py:116-121).  Every warp may call it; it is warp-uniform.
__device__ __forceinline__ int topk_with_ties(const uint64_t* sorted, int n, int K) {
  const int lane = threadIdx.x & 31;
  if (n == 0) return 0;
  const int kk = min(K, n);
  const uint32_t yk = uint32_t(sorted[kk - 1] >> 32);
  for (int j0 = kk; j0 < n; j0 += 32) {
    const unsigned b = __ballot_sync(kFull, j0 + lane < n && uint32_t(sorted[j0 + lane] >> 32) < yk);
    if (b) return j0 + __ffs(b) - 1;
  }
  return n;
}

// A greedy row's result: the id, or (vocab-parallel local step) a one-key
// record in which NaN sorts above every value.
__device__ __forceinline__ void write_greedy(const KArgs& a, int64_t row, int st, float b, int bi) {
  if (st != NS_OK) {
    a.out_ids[row] = int64_t(st);
  } else if (a.vp_keys) {
    const uint32_t hi = (b != b) ? 0xFFFFFFFFu : f2key(b + 0.0f);
    const uint32_t gid = uint32_t(int64_t(bi) + a.vocab_offset);
    a.vp_keys[row * a.vp_cap] = int64_t((uint64_t(hi) << 32) | uint64_t(~gid));
    a.out_ids[row] = 1;
  } else {
    a.out_ids[row] = int64_t(bi) + a.vocab_offset;
  }
}

// The end of a GREEDY, FAST or NUCLEUS row with few
// barriers.
// GREEDY: each CTA reduces its warps' (value, first index); a cluster's
// leader reads the CTAs' results in parallel.
// FAST / NUCLEUS: after every warp published its final bound, each warp turns
// its survivors of the tightest bound into keys (f2key(x / T) << 32) | ~id in
// its own stage bytes (its copies are all consumed); each warp places its keys
// in the CTA's union by counting the keys above them in all eight lists, into
// the candidate buffers (no longer read).  One CTA: finalize_keys takes the
// top-k with ties.  A cluster: each CTA keeps its own top-k with ties (which
// holds every element of the row's top-k that it owns), and the leader merges
// the CTAs' lists through distributed shared memory.
// Returns false (the same on every thread of the cluster) when the row
// continues on the general merge below: tied values that overflowed a buffer
// (multi-pass path), or a union of more than kRankMax survivors in one CTA
// (kMergeStage over a cluster's lists).
template <int DT>
__device__ bool row_tail(const Ctx<DT>& c, const KArgs& a, cg::cluster_group& cluster, int CL, int rank, int mode,
                         bool ok, const WarpCand& s, float best, int bidx, float topp) {
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = c.row;
  if (mode == MODE_GREEDY) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(kFull, best, o);
      const int oi = __shfl_xor_sync(kFull, bidx, o);
      if (better(ob, oi, best, bidx)) {
        best = ob;
        bidx = oi;
      }
    }
    if (lane == 0) {
      m->wbest[warp] = best;
      m->widx[warp] = bidx;
    }
    __syncthreads();
    if (tid == 0) {
      float b = m->wbest[0];
      int bi = m->widx[0];
      for (int w = 1; w < kWarps; ++w)
        if (better(m->wbest[w], m->widx[w], b, bi)) {
          b = m->wbest[w];
          bi = m->widx[w];
        }
      m->g_best = b;
      m->g_idx = bi;
      if (CL == 1) write_greedy(a, row, status_from_flags(m->flags, true), b, bi);
    }
    if (CL == 1) return true;
    cluster.sync();
    if (rank == 0 && warp == 0) {
      float b = -INFINITY;
      int bi = INT_MAX, fl = 0;
      if (lane < CL) {
        const Misc* rm = cluster.map_shared_rank(m, lane);
        b = rm->g_best;
        bi = rm->g_idx;
        fl = rm->flags;
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(kFull, b, o);
        const int oi = __shfl_xor_sync(kFull, bi, o);
        fl |= __shfl_xor_sync(kFull, fl, o);
        if (better(ob, oi, b, bi)) {
          b = ob;
          bi = oi;
        }
      }
      if (lane == 0) write_greedy(a, row, status_from_flags(fl, true), b, bi);
    }
    cluster.sync();  // the leader's reads are done before any CTA exits
    return true;
  }
  // every warp's final bound, then only survivors of the tightest become keys
  const bool nuc = (mode == MODE_NUCLEUS);
  if (nuc) {  // the row's largest scaled value, for its total mass
    const float ym = warp_row_max(c);
    if (lane == 0) m->wbest[warp] = ym;
  }
  if (ok) publish_bound(c, s);
  __syncthreads();
  WarpCand f = s;
  read_shared_tau(c, f);
  float M = -INFINITY;
  if (nuc) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m->wbest[w]);
    const double W = (M > -INFINITY) ? warp_row_mass(c, M) : 0.0;
    if (lane == 0) m->d_red[warp] = W;
  }
  uint64_t* keys = reinterpret_cast<uint64_t*>(c.stage(warp, 0));
  int nw = 0;
  if (ok && !s.ovf) {
    for (int i0 = 0; i0 < s.n; i0 += 32) {
      const int i = i0 + lane;
      const bool keep = i < s.n && s.x[i] >= f.tau;
      const unsigned mk = __ballot_sync(kFull, keep);
      if (keep) {
        const float y = __fdiv_rn(s.x[i], c.Tabs) + 0.0f;  // -0 and +0 tie
        keys[nw + __popc(mk & lanemask_lt())] = (uint64_t(f2key(y)) << 32) | uint64_t(~uint32_t(c.c0 + s.col[i]));
      }
      nw += __popc(mk);
    }
  }
  if (lane == 0) {
    if (nw & 1) keys[nw] = 0ull;  // pad to whole pairs
    m->wn[warp] = nw;
  }
  if (mode == MODE_WIDEK) {  // this warp's largest scaled value (the sort below may not run)
    uint64_t mk = 0;
    for (int i = lane; i < nw; i += 32) mk = max(mk, keys[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mk = max(mk, __shfl_xor_sync(kFull, mk, o));
    if (lane == 0) m->wbest[warp] = nw ? key2f(uint32_t(mk >> 32)) : -INFINITY;
  }
  __syncthreads();
  int n = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) n += m->wn[w];
  // A union past kRankMax: one CTA keeps its candidate buffers (no local sort)
  // for the radix-select merge; NUCLEUS rows and clusters (whose other CTAs
  // reuse their buffers for the sort) take the multi-pass path.
  if (n > kRankMax && tid == 0) atomicOr(&m->flags, (nuc || CL > 1) ? F_OVF : F_BIG);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(c.cx);
  if (n <= kRankMax) {
    for (int i = lane; i < nw; i += 32) {
      const uint64_t ki = keys[i];
      int pos = 0;
      for (int w2 = 0; w2 < kWarps; ++w2) {
        const uint64_t* k2 = reinterpret_cast<const uint64_t*>(c.stage(w2, 0));
        const int n2 = m->wn[w2];
#pragma unroll 4
        for (int j = 0; j < n2; j += 2) {
          const ulonglong2 p = *reinterpret_cast<const ulonglong2*>(k2 + j);
          pos += ((p.x > ki) ? 1 : 0) + ((p.y > ki) ? 1 : 0);
        }
      }
      sorted[pos] = ki;
    }
  }
  __syncthreads();
  if (CL == 1) {
    const int fl1 = m->flags;
    double Z = -1.0;
    if (nuc) {  // kept for the wide nucleus pass
      Z = 0.0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) Z += m->d_red[w];
      if (tid == 0) {
        m->nuc_M = M;
        m->nuc_Z = Z;
        m->nuc_yk = -INFINITY;
        m->nuc_cov = -1.0f;
      }
    }
    if (mode == MODE_WIDEK && !(fl1 & (F_NAN | F_TIMEOUT | F_BADID | F_HIST))) {
      // the kNucleusK largest give the row's largest value and the window scale
      if (tid == 0) {
        float Mw = -INFINITY;
        for (int w = 0; w < kWarps; ++w) Mw = fmaxf(Mw, m->wbest[w]);
        const bool have = !(fl1 & F_OVF) && n > 0;  // no candidate buffer overflowed
        m->nuc_M = have ? Mw : __int_as_float(0x7fc00000);  // NaN: unknown
        // the kNucleusK-th largest: from the sorted union, else the tightest bound (below it)
        m->nuc_yk = !have ? -INFINITY
                          : (n <= kRankMax && n >= c.K) ? key2f(uint32_t(sorted[c.K - 1] >> 32))
                                                        : __fdiv_rn(f.tau, c.Tabs);
        atomicOr(&m->flags, F_OVF);
      }
      __syncthreads();
      return false;
    }
    if ((fl1 & (F_OVF | F_BIG)) && !(fl1 & (F_NAN | F_TIMEOUT | F_BADID | F_HIST))) return false;
    const int st = status_from_flags(fl1, false);
    if (st != NS_OK) {
      if (tid == 0) a.out_ids[row] = st;
      return true;
    }
    if (nuc) {
      // the kNucleusK largest with ties must hold more than p of the row's
      // mass (with a margin above the sums' rounding), else a wider pass
      if (warp == 0) {
        const int nfin = topk_with_ties(sorted, n, c.K);
        double cm = 0.0;
        for (int j = lane; j < nfin; j += 32) cm += double(expf(__fsub_rn(key2f(uint32_t(sorted[j] >> 32)), M)));
#pragma unroll
        for (int o = 16; o; o >>= 1) cm += __shfl_xor_sync(kFull, cm, o);
        const bool covered = nfin > 0 && M > -INFINITY && cm > (double(topp) + 1e-6) * Z;
        if (lane == 0 && !covered) {
          atomicOr(&m->flags, F_OVF);
          if (n > 0) m->nuc_yk = key2f(uint32_t(sorted[min(c.K, n) - 1] >> 32));
          if (Z > 0.0) m->nuc_cov = float(cm / Z);
        }
      }
      __syncthreads();
      if (m->flags & F_OVF) return false;
    }
    finalize_keys(c, a, row, topp, sorted, n, n, Z);
    return true;
  }
  // ---- a cluster: this CTA's top-k with ties, then the leader merges ----
  if (warp == 0) {  // topk_with_ties is warp-synchronous: the whole warp computes it
    const int nf = topk_with_ties(sorted, min(n, kRankMax), c.K);
    if (lane == 0) m->n_merge = nf;
  }
  if (nuc && tid == 0) {  // this CTA's largest scaled value and its mass below it
    double Wc = 0.0;
    for (int w = 0; w < kWarps; ++w) Wc += m->d_red[w];
    m->c_M = M;
    m->c_W = Wc;
  }
  cluster.sync();
  int fl_all = 0, n_all = 0;
  for (int r = 0; r < CL; ++r) {
    const Misc* rm = cluster.map_shared_rank(m, r);
    fl_all |= rm->flags;
    n_all += rm->n_merge;
  }
  const bool hard = (fl_all & (F_NAN | F_TIMEOUT | F_BADID | F_HIST)) != 0;
  // the lists are staged whole (kMergeStage keys) and the first kRankMax
  // positions of their union placed; a tie run past them overflows
  if (!hard && ((fl_all & F_OVF) || n_all > kMergeStage)) {  // the multi-pass path, uniformly
    cluster.sync();
    if (tid == 0) atomicOr(&m->flags, F_OVF);
    __syncthreads();
    return false;
  }
  uint64_t* lists = reinterpret_cast<uint64_t*>(c.stages);
  uint64_t* gsorted = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff) + kRankMax;
  int total = 0;
  if (rank == 0 && !hard) {
    if (tid == 0) {
      int t = 0;
      for (int r = 0; r < CL; ++r) {
        m->roff[r] = t;
        t += cluster.map_shared_rank(m, r)->n_merge;
      }
      m->roff[CL] = t;
    }
    __syncthreads();
    total = m->roff[CL];
    for (int r = warp; r < CL; r += kWarps) {
      const uint64_t* src = reinterpret_cast<const uint64_t*>(cluster.map_shared_rank(c.cx, r));
      for (int i = m->roff[r] + lane; i < m->roff[r + 1]; i += 32) lists[i] = src[i - m->roff[r]];
    }
  }
  cluster.sync();  // the leader's reads are done before any CTA exits
  if (!hard && (n_all > kRankMax || nuc)) {
    // The same decision on every CTA: the leader places the first kRankMax
    // positions and checks that the tie run at the k-th ends inside them
    // (NUCLEUS: and that the candidates hold more than p of the row's mass,
    // rebuilt from the CTAs' maxima and masses); if not, the whole cluster
    // takes the multi-pass path.
    const int np = min(n_all, kRankMax);
    if (rank == 0) {
      place_sorted_lists(lists, m->roff, CL, total, gsorted);
      if (warp == 0) {  // warp-synchronous
        const int nf = topk_with_ties(gsorted, np, c.K);
        bool good = !(nf >= np && n_all > np);
        if (nuc) {
          float Mg = -INFINITY;
          for (int r = 0; r < CL; ++r) Mg = fmaxf(Mg, cluster.map_shared_rank(m, r)->c_M);
          double Z = 0.0;
          for (int r = 0; r < CL; ++r) {
            const Misc* rm = cluster.map_shared_rank(m, r);
            if (rm->c_M > -INFINITY) Z += rm->c_W * double(expf(__fsub_rn(rm->c_M, Mg)));
          }
          double cm = 0.0;
          for (int j = lane; j < nf; j += 32) cm += double(expf(__fsub_rn(key2f(uint32_t(gsorted[j] >> 32)), Mg)));
#pragma unroll
          for (int o = 16; o; o >>= 1) cm += __shfl_xor_sync(kFull, cm, o);
          good = good && nf > 0 && Mg > -INFINITY && key2f(uint32_t(gsorted[0] >> 32)) == Mg &&
                 cm > (double(topp) + 1e-6) * Z;
          if (lane == 0) m->nuc_Z = Z;
        }
        if (lane == 0) m->n_merge = good ? nf : -1;
      }
    }
    cluster.sync();
    const bool over = cluster.map_shared_rank(m, 0)->n_merge < 0;
    cluster.sync();  // the leader's verdict is read before any CTA moves on
    if (over) {
      if (tid == 0) atomicOr(&m->flags, F_OVF);
      __syncthreads();
      return false;
    }
    if (rank == 0) finalize_keys(c, a, row, topp, gsorted, np, n_all, nuc ? m->nuc_Z : -1.0);
    return true;
  }
  if (rank != 0) return true;
  if (hard) {
    if (tid == 0) a.out_ids[row] = status_from_flags(fl_all, false);
    return true;
  }
  place_sorted_lists(lists, m->roff, CL, total, gsorted);
  finalize_keys(c, a, row, topp, gsorted, total, total);
  return true;
}

// SOFTMAX / NUCLEUS, after the stream (tile masses in place, penalised
// history values computed): this warp's largest scaled value over its tiles
// and its history columns (NaN or +inf there flags F_NAN), warp-uniform ...
template <int DT>
__device__ __forceinline__ float warp_row_max(const Ctx<DT>& c) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* tY = softmax_tile_max(c);
  float ymax = -INFINITY;
  bool bad = false;
  for (int t = lane; t < c.wtiles(warp); t += 32) ymax = fmaxf(ymax, tY[warp * c.tpw + t]);
  if (c.pen)
    for (int r = c.m->segoff[warp] + lane; r < c.m->segoff[warp + 1]; r += 32) {
      const float y = __fdiv_rn(c.pval[r], c.Tabs);
      bad |= (y != y) || y == INFINITY;
      ymax = fmaxf(ymax, y);
    }
  if (__any_sync(kFull, bad) && lane == 0) atomicOr(&c.m->flags, F_NAN);
#pragma unroll
  for (int o = 16; o; o >>= 1) ymax = fmaxf(ymax, __shfl_xor_sync(kFull, ymax, o));
  return ymax;
}

// ... and this warp's mass with the row's largest scaled value M: tile masses
// times expf(ym_t - M) plus expf(y - M) of its history columns (float64).
template <int DT>
__device__ __forceinline__ double warp_row_mass(const Ctx<DT>& c, float M) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const double* tD = softmax_tile_mass(c.tacc);
  const float* tY = softmax_tile_max(c);
  double W = 0.0;
  for (int t = lane; t < c.wtiles(warp); t += 32) {
    const float y = tY[warp * c.tpw + t];
    if (y > -INFINITY) W += tD[warp * c.tpw + t] * double(expf(__fsub_rn(y, M)));
  }
  if (c.pen)
    for (int r = c.m->segoff[warp] + lane; r < c.m->segoff[warp + 1]; r += 32) {
      const float y = __fdiv_rn(c.pval[r], c.Tabs);
      if (y > -INFINITY) W += double(expf(__fsub_rn(y, M)));
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) W += __shfl_xor_sync(kFull, W, o);
  return W;
}

// SOFTMAX rows: after the stream (tile masses in place, penalised history
// values computed), locate the draw u * Z in column order -- CTA of the
// cluster, warp, then tile -- and read that tile again to find the id.
// Weights are expf(rn(x / |T|) - ym_t) * expf(ym_t - M) for the tiles' values
// and expf(rn(xp / |T|) - M) for history columns (penalised xp), summed in
// float64 in the same way for the totals and for the final scan.  A cluster
// exchanges each CTA's largest value and mass through distributed shared
// memory (three cluster barriers on every path).
template <int DT>
__device__ void softmax_tail(const Ctx<DT>& c, const KArgs& a, uint64_t policy, cg::cluster_group& cluster, int CL,
                             int rank) {
  using E = Elem<DT>;
  using R = typename E::raw;
  constexpr int TE = Ctx<DT>::TE;
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = c.row;
  const double* tD = softmax_tile_mass(c.tacc);
  const float* tY = softmax_tile_max(c);
  const int nt = c.wtiles(warp);
  auto hist_y = [&](int r) { return __fdiv_rn(c.pval[r], c.Tabs); };

  // 1. the row's largest scaled value
  const float ymax = warp_row_max(c);
  if (lane == 0) m->wbest[warp] = ymax;
  __syncthreads();
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m->wbest[w]);
  int fl = m->flags;
  if (CL > 1) {
    if (tid == 0) m->c_M = M;
    cluster.sync();
    M = -INFINITY;
    fl = 0;
    for (int r = 0; r < CL; ++r) {
      const Misc* rm = cluster.map_shared_rank(m, r);
      M = fmaxf(M, rm->c_M);
      fl |= rm->flags;
    }
  }
  const int st = status_from_flags(fl, false);
  if (st != NS_OK || !(M > -INFINITY)) {  // the same decision on every CTA
    if (CL > 1) cluster.sync();           // every CTA has read the others
    if (rank == 0 && tid == 0) a.out_ids[row] = (st != NS_OK) ? st : NS_ERR_INVALID_DISTRIBUTION;
    return;
  }
  auto tile_scale = [&](int t) {
    const float y = tY[warp * c.tpw + t];
    return y > -INFINITY ? double(expf(__fsub_rn(y, M))) : 0.0;
  };

  // 2. this warp's mass, and this CTA's
  const double W = warp_row_mass(c, M);
  if (lane == 0) m->d_red[warp] = W;
  __syncthreads();
  if (tid == 0) {
    double Wc = 0.0;
    for (int w = 0; w < kWarps; ++w) Wc += m->d_red[w];
    m->c_W = Wc;
  }
  if (CL > 1)
    cluster.sync();
  else
    __syncthreads();

  // 3. the CTA, then the warp holding u * Z (the last with mass if rounding
  // leaves the target past the end); every CTA computes the same choice
  if (tid == 0) {
    const float u = a.uniforms ? c.u_pre : philox_uniform(a.seed, a.offset, uint64_t(row));
    double Z = 0.0;
    for (int r = 0; r < CL; ++r) Z += cluster.map_shared_rank(m, r)->c_W;
    double target = double(u) * Z;
    int rs = -1, rlast = 0;
    double rbefore = 0.0;
    for (int r = 0; r < CL; ++r) {
      const double Wr = cluster.map_shared_rank(m, r)->c_W;
      if (Wr > 0.0) rlast = r;
      if (rs < 0 && rbefore + Wr > target) rs = r;
      if (rs < 0) rbefore += Wr;
    }
    if (rs < 0) {
      rs = rlast;
      rbefore = Z - cluster.map_shared_rank(m, rlast)->c_W;
    }
    m->s_rank = rs;
    target -= rbefore;  // inside CTA rs
    double before = 0.0;
    int sw = -1, last = 0;
    for (int w = 0; w < kWarps; ++w) {
      if (m->d_red[w] > 0.0) last = w;
      if (sw < 0 && before + m->d_red[w] > target) sw = w;
      if (sw < 0) before += m->d_red[w];
    }
    if (sw < 0) {
      sw = last;
      before = Z - m->d_red[last];
    }
    m->s_warp = sw;
    m->s_rem = target - before;
  }
  if (CL > 1) cluster.sync();  // every CTA has read the others
  __syncthreads();
  if (rank != m->s_rank || warp != m->s_warp) return;

  // 4. the tile: per-tile totals (scaled tile mass + its history columns),
  // scanned in column order 32 tiles at a time
  double rem = m->s_rem;
  int ts = -1, tlast = 0;
  for (int t0 = 0; t0 < nt && ts < 0; t0 += 32) {
    const int t = t0 + lane;
    double T = 0.0;
    if (t < nt) {
      T = tD[warp * c.tpw + t] * tile_scale(t);
      if (c.pen) {
        const int2 rr = tile_ranks(c, warp, t);
        for (int r = rr.x; r < rr.y; ++r) {
          const float y = hist_y(r);
          if (y > -INFINITY) T += double(expf(__fsub_rn(y, M)));
        }
      }
    }
    double incl = T;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    const unsigned hit = __ballot_sync(kFull, t < nt && incl > rem);
    const unsigned nz = __ballot_sync(kFull, t < nt && T > 0.0);
    if (nz) tlast = t0 + 31 - __clz(nz);
    if (hit) {
      const int l = __ffs(hit) - 1;
      ts = t0 + l;
      rem -= __shfl_sync(kFull, incl - T, l);
    } else {
      rem -= __shfl_sync(kFull, incl, 31);
    }
  }
  if (ts < 0) {  // rounding left the target past the last tile: its last element
    ts = tlast;
    rem = INFINITY;
  }

  // 5. read tile ts again and scan it in column order, 32 consecutive
  // elements per round (one per lane); history columns take their penalised
  // values
  const int sidx = 0;
  const uint32_t parity = uint32_t((nt + 1) / 2) & 1u;  // phases stage 0 completed in the stream
  if (lane == 0) issue_tile(c, warp, ts, sidx, policy);
  if (!__all_sync(kFull, mbar_wait_bounded(c.sbar(warp, sidx), parity))) {
    if (lane == 0) a.out_ids[row] = NS_ERR_DEVICE_TIMEOUT;
    return;
  }
  __syncwarp();  // lane 0's plain-load head / tail
  const R* sr = reinterpret_cast<const R*>(c.stage(warp, sidx));
  const int len = c.tile_len(warp, ts), lead = c.tile_lead(warp, ts);
  const int base = warp * c.pw + ts * TE;  // CTA-relative column of element 0
  const float ym = tY[warp * c.tpw + ts];
  const double f = tile_scale(ts);
  int2 rr = make_int2(0, 0);
  if (c.pen) rr = tile_ranks(c, warp, ts);
  int pick = -1, lastnz = -1;
  for (int e0 = 0; e0 < len; e0 += 32) {
    const int e = e0 + lane;
    double wgt = 0.0;
    if (e < len) {
      int hr = -1;
      for (int r = rr.x; r < rr.y; ++r)
        if (c.colr[r] - base == e) hr = r;
      if (hr >= 0) {
        const float y = hist_y(hr);
        if (y > -INFINITY) wgt = double(expf(__fsub_rn(y, M)));
      } else {
        const float x = c.neg ? -E::widen(sr[lead + e]) : E::widen(sr[lead + e]);
        if (ym > -INFINITY) wgt = double(softmax_weight(x, ym, c.Tabs, __frcp_rn(c.Tabs))) * f;
      }
    }
    double incl = wgt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += v;
    }
    const unsigned nz = __ballot_sync(kFull, wgt > 0.0);
    if (nz) lastnz = e0 + 31 - __clz(nz);
    const unsigned hit = __ballot_sync(kFull, wgt > 0.0 && incl > rem);
    if (hit) {
      pick = e0 + __ffs(hit) - 1;
      break;
    }
    rem -= __shfl_sync(kFull, incl, 31);
  }
  if (pick < 0) pick = lastnz;  // rounding left the target past the end: the last weighted element
  if (lane == 0)
    a.out_ids[row] = (pick >= 0) ? int64_t(c.c0 + base + pick) + a.vocab_offset : NS_ERR_INVALID_DISTRIBUTION;
}

// Leader, FAST rows: the K-th largest value over the union of every warp list
// of every CTA in the cluster (read through distributed shared memory), then
// the survivors rn(x / T) >= rn(x_K / T) into the merge area.  Up to
// kThreads * kMergeReg entries are held in registers and selected bit by bit
// (one block count per bit); larger unions use the shared-memory radix select.
constexpr int kMergeReg = 16;

template <int DT>
__device__ __forceinline__ void leader_gather(const Ctx<DT>& c, const KArgs& a, cg::cluster_group& cluster, int CL) {
  Misc* m = c.m;
  const int tid = threadIdx.x;
  const int nl = CL * kWarps;
  const int tot = m->roff[nl];
  auto owner = [&](int gi) {
    int lo = 0, hi = nl - 1;  // last list l with roff[l] <= gi
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (m->roff[mid] <= gi)
        lo = mid;
      else
        hi = mid - 1;
    }
    return lo;
  };
  float* my = reinterpret_cast<float*>(c.stages);
  int* mid = reinterpret_cast<int*>(c.stages + size_t(a.merge_cap) * 4);
  if (tot <= kThreads * kMergeReg) {
    uint32_t key[kMergeReg];
    int col[kMergeReg];
#pragma unroll
    for (int q = 0; q < kMergeReg; ++q) {
      const int gi = q * kThreads + tid;
      key[q] = 0u;
      col[q] = 0;
      if (gi < tot) {
        const int l = owner(gi);
        const int r = l / kWarps, idx = (l % kWarps) * kCapW + gi - m->roff[l];
        key[q] = f2key(cluster.map_shared_rank(c.cx, r)[idx]);
        col[q] = cluster.map_shared_rank(c.cid, r)[idx] + m->rc0[r];
      }
    }
    float thr = -INFINITY;
    uint32_t kk = 0;
    if (tot > c.K && block_kth_regs(m, key, c.K, &kk)) thr = __fdiv_rn(key2f(kk), c.Tabs);
#pragma unroll
    for (int q = 0; q < kMergeReg; ++q) {
      if (key[q] == 0u) continue;
      const float y = __fdiv_rn(key2f(key[q]), c.Tabs);
      if (y >= thr) {
        const int pos = atomicAdd(&m->n_merge, 1);
        if (pos < a.merge_cap) {
          my[pos] = y;
          mid[pos] = col[q];
        }
      }
    }
  } else {
    uint32_t key = 0;
    const bool have = (tot > c.K) && block_radix_kth(
                                         m, c.K,
                                         [&](auto f) {
                                           for (int gi = tid; gi < tot; gi += kThreads) {
                                             const int l = owner(gi);
                                             const float* rcx =
                                                 cluster.map_shared_rank(c.cx, l / kWarps) + (l % kWarps) * kCapW;
                                             f(rcx[gi - m->roff[l]]);
                                           }
                                         },
                                         &key);
    const float thr = have ? __fdiv_rn(key2f(key), c.Tabs) : -INFINITY;
    for (int gi = tid; gi < tot; gi += kThreads) {
      const int l = owner(gi);
      const int r = l / kWarps, wl = l % kWarps;
      const float* rcx = cluster.map_shared_rank(c.cx, r) + wl * kCapW;
      const int* rcid = cluster.map_shared_rank(c.cid, r) + wl * kCapW;
      const float y = __fdiv_rn(rcx[gi - m->roff[l]], c.Tabs);
      if (y >= thr) {
        const int pos = atomicAdd(&m->n_merge, 1);
        if (pos < a.merge_cap) {
          my[pos] = y;
          mid[pos] = rcid[gi - m->roff[l]] + m->rc0[r];
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0 && m->n_merge > a.merge_cap) {
    m->flags |= F_OVF;
    a.out_ids[c.row] = NS_ERR_CANDIDATE_OVERFLOW;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// GENERAL rows: top-k disabled, top-k > kFastK, or ties that overflowed the
// FAST buffers.  Every CTA of the cluster streams its columns several times
// (the row is re-read), and cluster-wide reductions go through distributed
// shared memory.  y = rn(x / T) is computed exactly for every value.
// Probability masses exp(y - M) are accumulated in 2^-40 fixed point, so all
// sums (histogram bins, tile sums, the final ordered scan) are exact and
// mutually consistent.
//
//   P1      max of x; NaN/+inf check; 11-bit count histogram if top-k is on
//   P2, P3  count histograms of the next 11 and 10 bits: the exact K-th value
//   P4      Z = sum exp(y - M) over the top-k survivors, per-tile masses, and
//           an 11-bit mass histogram of y if top-p is on
//   P5, P6  mass histograms of the next bits: the value c at which the
//           descending cumulative mass first exceeds p * Z, the mass above it
//           and the number of ties at c (reference sampler.py:122-131)
//   P7      per-tile kept mass (y > c, plus the first ties at c in id order)
//   P8      the warp owning the tile that holds u * total reloads it and
//           scans it in id order
// ---------------------------------------------------------------------------
constexpr int kGBins = 2048;                      // 11-bit digits
constexpr double kFx = 1099511627776.0;           // 2^40: sums stay below 2^64 for vocab <= 2^24

__device__ __forceinline__ unsigned long long to_fx(float e) {
  return (unsigned long long)(double(e) * kFx);
}

// A bound below every x (same domain) with rn(x / Tabs) >= ylo: ylo * Tabs
// less a relative margin far above one quotient rounding and an absolute one
// above the subnormal spacing (a pass's 16-byte-group skip; -inf: none).
__device__ __forceinline__ float x_floor_of_y(float ylo, float Tabs) {
  if (!(ylo > -INFINITY)) return -INFINITY;  // -inf or NaN: no bound
  const double b = double(ylo) * double(Tabs);
  return __double2float_rd(b - fabs(b) * 0x1p-20 - double(Tabs) * 0x1p-120);
}

// One pass of this warp over its tiles: fe(x, col) for every value (x in the
// negated domain when T < 0, col CTA-relative), ft(t) after each tile (all
// lanes).  `seq` counts the copies this warp has made (it selects ring slots
// and barrier phases across passes); `pre_issued` tiles were issued already.
// gmin: the 16-byte groups whose values are all below it (in that domain)
// are skipped -- fe must ignore every such value.  Each lane then marks its
// groups that reach gmin and the warp works through them one group per lane
// per round, so a sparse set of hot groups costs a few rounds, not a full
// divergent sweep.
template <int DT, class FElem, class FTile>
__device__ __forceinline__ bool warp_pass(const Ctx<DT>& c, int& seq, int pre_issued, uint64_t policy, float rep,
                                          float pres, float freq, FElem fe, FTile ft, float gmin = -INFINITY) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = c.wtiles(w);
  const int s0 = seq;
  if (lane == 0)
    for (int t = pre_issued; t < min(kWStages, nt); ++t) issue_tile(c, w, t, (s0 + t) % kWStages, policy);
  for (int t = 0; t < nt; ++t) {
    const int sq = s0 + t;
    const int sidx = sq % kWStages;
    const bool ok = __all_sync(kFull, mbar_wait_bounded(c.sbar(w, sidx), uint32_t(sq / kWStages) & 1u));
    if (!ok) {
      if (lane == 0) {
        atomicOr(&c.m->flags, F_TIMEOUT);
        for (int u = t; u < min(nt, t + kWStages); ++u)
          mbar_wait_bounded(c.sbar(w, (s0 + u) % kWStages), uint32_t((s0 + u) / kWStages) & 1u);
      }
      __syncwarp();
      seq = s0 + nt;
      return false;
    }
    uint8_t* st = c.stage(w, sidx);
    patch_tile(c, w, t, st, [&](bool has, float xp, int col) {
      if (has) fe(xp, col);
    });
    __syncwarp();
    const int len = c.tile_len(w, t), lead = c.tile_lead(w, t);
    const int n_groups = (lead + len + VE - 1) / VE;
    const int colbase = w * c.pw + t * TE - lead;
    if (gmin > -INFINITY) {
      unsigned gm = 0;  // bit k: group k * 32 + lane reaches gmin (or holds NaN)
      for (int k = 0; k * 32 + lane < n_groups; ++k) {
        const uint4 v = *reinterpret_cast<const uint4*>(st + (k * 32 + lane) * 16);
        const float gx = c.neg ? group_extreme<DT, true>(v) : group_extreme<DT, false>(v);
        gm |= (gx < gmin ? 0u : 1u) << k;
      }
      while (__any_sync(kFull, gm != 0u)) {
        if (gm) {
          const int q = (__ffs(gm) - 1) * 32 + lane;
          gm &= gm - 1u;
          float x[VE];
          unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
          for (int i = 0; i < VE; ++i) {
            const int e = q * VE + i;
            if (e >= lead && e < lead + len) fe(c.neg ? -x[i] : x[i], colbase + e);
          }
        }
      }
    } else {
      for (int q = lane; q < n_groups; q += 32) {
        float x[VE];
        unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
        for (int i = 0; i < VE; ++i) {
          const int e = q * VE + i;
          if (e >= lead && e < lead + len) fe(c.neg ? -x[i] : x[i], colbase + e);
        }
      }
    }
    ft(t);
    __syncwarp();
    if (lane == 0 && t + kWStages < nt) issue_tile(c, w, t + kWStages, (s0 + t + kWStages) % kWStages, policy);
  }
  seq = s0 + nt;
  return true;
}

__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Digit search over a histogram of nb bins held by every CTA of the cluster
// at the same shared-memory address (combined through DSMEM, ranks in order):
// scanning from the highest bin, the first bin whose inclusive cumulative
// value is >= target (strict: > target).  Sets m->g_bin (-1: never) and
// m->g_before (cumulative value of the bins above it).  Exact integer sums.
__device__ void cluster_digit(cg::cluster_group& cl, int CL, Misc* m, const unsigned long long* h, int nb,
                              unsigned long long target, bool strict) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = nb / kThreads;  // 8 or 4 bins per thread, highest bins first
  unsigned long long v[kGBins / kThreads];
  unsigned long long local = 0;
#pragma unroll
  for (int k = 0; k < kGBins / kThreads; ++k) {
    v[k] = 0;
    if (k < per) {
      const int b = nb - 1 - (tid * per + k);
      for (int r = 0; r < CL; ++r) v[k] += cl.map_shared_rank(const_cast<unsigned long long*>(h), r)[b];
      local += v[k];
    }
  }
  unsigned long long incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += t;
  }
  if (tid == 0) m->g_bin = -1;
  if (lane == 31) m->g_sum[warp] = incl;
  __syncthreads();
  unsigned long long run = incl - local;
  for (int w = 0; w < warp; ++w) run += m->g_sum[w];
#pragma unroll
  for (int k = 0; k < kGBins / kThreads; ++k) {
    if (k < per) {
      const unsigned long long prev = run;
      run += v[k];
      const bool was = strict ? prev > target : prev >= target;
      const bool now = strict ? run > target : run >= target;
      if (!was && now) {
        m->g_bin = nb - 1 - (tid * per + k);
        m->g_before = prev;
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// NUCLEUS rows (one CTA) whose nucleus is larger than the kNucleusK
// candidates.  One more pass over the row counts the values within D nats of
// M in 255 bins of D / 255 nats (d = M - x / |T| through a reciprocal; deeper
// values, and 16-byte groups holding only such values, are skipped) and
// collects those of the first kb bins as keys (f2key(y) << 32 | ~id, y =
// rn(x / |T|)).  M, Z: the row's largest scaled value and total mass from the
// stream; D = dk + 4.5 and the keys' window dk + 3.5 nats, dk the
// kNucleusK-th largest value's distance from M.  On the first pass a value in
// bin b weighs at least e^-(b+1) D / 255 (less a margin for the rounding), so
// the smallest bin prefix whose guaranteed mass exceeds (p + 1e-6) Z holds
// the nucleus; later passes (a window twice as wide, or the same one when the prefix
// holds more values than the keys) sum each bin's masses (float) instead.  A prefix past the keys' bins, or more than kWideCap keys: one more
// pass collects that prefix alone; a prefix past kWideCap values: the large
// nucleus path (nucleus_big) with the bin where the exact mass crosses p Z.
// The collected set is an upper set of x, so every value scaled above its
// smallest y is in it; the keys are sorted (by bucket of y, then rank), and
// when those values alone hold more than (p + 1e-6) Z (float64 sums) the
// top-p cut lies before the smallest y: the cut and the draw run on the keys
// with Z as the softmax normaliser (reference sampler.py:122-131, 86-89).
// Returns false -- the same on every thread -- when the row continues on the
// multi-pass path; true when its result is written.
// ---------------------------------------------------------------------------
constexpr int kWideBins = kBins;  // 255 window bins + the deeper values
constexpr float kWideMaxNats = 32.0f;
constexpr int kWideCap = kCandBytes / 8;  // keys held by the candidate buffers
static_assert(kWideBins == kThreads, "one bin per thread in the prefix scan");
static_assert(size_t(kMergeCap + kWideCap) * 8 <= kRankKeysOff + size_t(kRankMax) * 8,
              "the bucket staging ends where the sorted keys start");
static_assert(kRankKeysOff + size_t(kRankMax + kWideCap) * 8 <= size_t(kStageBytes),
              "the sorted window keys fit the stage area");

__device__ __forceinline__ int wide_bin(float x, float M, float r, float S) {
  // explicit roundings: every pass bins a value identically
  const float d = __fmul_rn(__fsub_rn(M, __fmul_rn(x, r)), S);
  return d < float(kWideBins - 1) ? int(fmaxf(d, 0.0f)) : kWideBins - 1;
}

// A value below this bound lies at least dd nats below M: (M - dd) |T| less
// a margin far above the few roundings of wide_bin's reciprocal quotient.
__device__ __forceinline__ float wide_floor(float M, float dd, float Tabs) {
  const float b = (M - dd) * Tabs;
  return b - (fabsf(M) + dd) * Tabs * 0x1p-18f - 1e-30f;
}

// The bins of the ends of y's class -- every x (the pass's domain) with
// rn(x / Tabs) == y -- found by walking the float grid from y * Tabs: *blo
// for its largest x, *bhi for its smallest.  False (unsure) when a walk takes
// more than 64 steps or y has no such x.
__device__ bool y_class_bins(float y, float Tabs, float M, float r, float S, int* blo, int* bhi) {
  auto yq = [&](float x) { return __fdiv_rn(x, Tabs) + 0.0f; };
  float x = y * Tabs;
  for (int i = 0; i < 64 && yq(x) < y; ++i) x = nextafterf(x, INFINITY);
  for (int i = 0; i < 64 && yq(x) > y; ++i) x = nextafterf(x, -INFINITY);
  if (yq(x) != y) return false;
  float lo = x, hi = x;
  int i = 0;
  for (; i < 64; ++i) {
    const float nx = nextafterf(lo, -INFINITY);
    if (yq(nx) != y) break;
    lo = nx;
  }
  if (i == 64) return false;
  for (i = 0; i < 64; ++i) {
    const float nx = nextafterf(hi, INFINITY);
    if (yq(nx) != y) break;
    hi = nx;
  }
  if (i == 64) return false;
  *blo = wide_bin(hi, M, r, S);
  *bhi = wide_bin(lo, M, r, S);
  return true;
}

// Whether every x with rn(x / Tabs) == y falls in bin jb.
__device__ bool y_class_in_bin(float y, float Tabs, float M, float r, float S, int jb) {
  int blo = 0, bhi = 0;
  return y_class_bins(y, Tabs, M, r, S, &blo, &bhi) && blo == jb && bhi == jb;
}

// NUCLEUS rows whose nucleus holds more values than the keys fit (one CTA):
// the window's bin jb holds the cut.  One more pass sums the exact masses of
// bins < jb per tile (2^-40 fixed point, as the multi-pass path) and collects
// bin jb alone as keys; the sorted keys give the cut (keep position j while
// the mass before it is at most p Z, reference sampler.py:122-131), the kept
// keys are added to their tiles, and the draw locates its tile and scans it
// again in id order (a value is kept iff its bin is below jb, or it is in bin
// jb with a key at or above the last kept key).  Returns false (the same on
// every thread) when the row continues on the multi-pass path: bin jb over
// kWideCap values, the exact mass of bins < jb already past p Z, or values
// tied with the cut that may lie in a neighbouring bin.
template <int DT>
__device__ bool nucleus_big(const Ctx<DT>& c, const KArgs& a, int& seq, uint64_t policy, float topp, float M,
                            double Z, float r, float S, int jb) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t* keys = reinterpret_cast<uint64_t*>(c.cx);
  unsigned long long* tmass = reinterpret_cast<unsigned long long*>(c.tacc);
  auto yof = [&](float x) { return __fdiv_rn(x, c.Tabs) + 0.0f; };  // -0 and +0 tie
  auto wfx = [&](float y) { return to_fx(expf(__fsub_rn(y, M))); };
  auto key_of = [&](float x, int col) {
    return (uint64_t(f2key(yof(x))) << 32) | uint64_t(~uint32_t(c.c0 + col));
  };
  if (tid == 0) m->w_n = 0;
  __syncthreads();
  {
    unsigned long long acc = 0;
    warp_pass(
        c, seq, 0, policy, c.rep, c.pres, c.freq,
        [&](float x, int col) {
          if (!(x > -INFINITY)) return;
          const int b = wide_bin(x, M, r, S);
          if (b < jb) {
            acc += wfx(yof(x));
          } else if (b == jb) {
            const int i = atomicAdd(&m->w_n, 1);
            if (i < kWideCap) keys[i] = key_of(x, col);
          }
        },
        [&](int t) {
          const unsigned long long sum = warp_sum_u64(acc);
          acc = 0;
          if (lane == 0) tmass[warp * c.tpw + t] = sum;
        },
        wide_floor(M, float(jb + 1) / S, c.Tabs));
  }
  __syncthreads();
  if (m->flags & F_TIMEOUT) {
    if (tid == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
    return true;
  }
  const int n = m->w_n;
  if (n > kWideCap || n == 0) return false;
  // the exact mass of bins < jb
  auto block_sum_u64 = [&](unsigned long long v) {
    v = warp_sum_u64(v);
    if (lane == 0) m->g_sum[warp] = v;
    __syncthreads();
    unsigned long long t = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += m->g_sum[w];
    __syncthreads();
    return t;
  };
  auto tile_sum = [&]() {
    unsigned long long v = 0;
    for (int w = 0; w < kWarps; ++w)
      for (int t = tid; t < c.wtiles(w); t += kThreads) v += tmass[w * c.tpw + t];
    return block_sum_u64(v);
  };
  const unsigned long long A = tile_sum();
  // bin jb's keys in descending order (sub-buckets of the bin by scaled value)
  uint64_t* tmp = reinterpret_cast<uint64_t*>(c.stages + size_t(kMergeCap) * 8);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff) + kRankMax;
  bucket_sort(
      m, keys, n, tmp, sorted,
      [&](uint64_t k) {
        const float d = ((M - key2f(uint32_t(k >> 32))) * S - float(jb)) * float(kBins - 1);
        return d < float(kBins - 1) ? int(fmaxf(d, 0.0f)) : kBins - 1;
      },
      [](uint64_t x, uint64_t y) { return x > y; });
  // the cut: L = the first position whose preceding mass exceeds p Z
  const unsigned long long target = (unsigned long long)(double(topp) * (Z * kFx));
  if (warp == 0) {
    const int per = (n + 31) / 32;
    const int i0 = min(lane * per, n), i1 = min(i0 + per, n);
    unsigned long long loc = 0;
    for (int i = i0; i < i1; ++i) loc += wfx(key2f(uint32_t(sorted[i] >> 32)));
    unsigned long long ex = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long v = __shfl_up_sync(kFull, ex, o);
      if (lane >= o) ex += v;
    }
    ex -= loc;
    unsigned long long cum = A + ex;
    int first = INT_MAX;
    for (int i = i0; i < i1 && first == INT_MAX; ++i) {
      if (cum > target) first = i;
      cum += wfx(key2f(uint32_t(sorted[i] >> 32)));
    }
    first = int(__reduce_min_sync(kFull, unsigned(first)));
    if (lane == 0) {
      const int L = first;  // kept: sorted[0, L)
      // the values tied with the last kept one must all lie in bin jb
      const bool ok = L >= 1 && L < n && y_class_in_bin(key2f(uint32_t(sorted[L - 1] >> 32)), c.Tabs, M, r, S, jb);
      m->w_L = ok ? L : -1;
      m->w_keyL = ok ? sorted[L - 1] : 0ull;
    }
  }
  __syncthreads();
  const int L = m->w_L;
  const uint64_t keyL = m->w_keyL;
  if (L < 0) return false;
  // kept keys by ascending id, their masses added to their tiles
  {
    uint64_t* byid = reinterpret_cast<uint64_t*>(c.stages);
    for (int i = tid; i < L; i += kThreads) {
      const uint64_t k = sorted[i];
      tmp[i] = (uint64_t(~uint32_t(k)) << 32) | (k >> 32);  // (id, y key)
    }
    __syncthreads();
    int sh = 0;
    while ((int64_t(c.c1) - 1) >> (8 + sh)) ++sh;  // call-local ids < c1
    bucket_sort(
        m, tmp, L, sorted, byid, [&](uint64_t k) { return int(uint32_t(k >> 32) >> sh); },
        [](uint64_t x, uint64_t y) { return x < y; });
    auto lower = [&](uint32_t id) {  // first kept key with id >= id
      int lo = 0, hi = L;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (uint32_t(byid[mid] >> 32) < id)
          lo = mid + 1;
        else
          hi = mid;
      }
      return lo;
    };
    for (int w = 0; w < kWarps; ++w)
      for (int t = tid; t < c.wtiles(w); t += kThreads) {
        const uint32_t col0 = uint32_t(c.c0 + w * c.pw + t * TE);
        const int i0 = lower(col0), i1 = lower(col0 + uint32_t(c.tile_len(w, t)));
        unsigned long long add = 0;
        for (int i = i0; i < i1; ++i) add += wfx(key2f(uint32_t(byid[i])));
        tmass[w * c.tpw + t] += add;
      }
  }
  __syncthreads();
  const unsigned long long W = tile_sum();
  // the tile holding u * W (the last kept tile if rounding leaves it past the end)
  const float u = a.uniforms ? c.u_pre : philox_uniform(a.seed, a.offset, uint64_t(c.row));
  const unsigned long long tgt = (unsigned long long)(double(u) * double(W));
  if (tid == 0) {
    int tsel = -1, tlast = -1;
    unsigned long long before = 0, run = 0;
    for (int w = 0; w < kWarps; ++w)
      for (int t = 0; t < c.wtiles(w); ++t) {
        const int gt = w * c.tpw + t;
        if (tmass[gt] > 0) tlast = gt;
        if (tsel < 0 && run + tmass[gt] > tgt) {
          tsel = gt;
          before = run;
        }
        run += tmass[gt];
      }
    m->g_bin = 0;
    if (tsel < 0) {
      tsel = tlast;
      m->g_bin = 1;
    }
    m->g_tile = tsel;
    m->g_tbefore = before;
  }
  __syncthreads();
  const int gsel = m->g_tile;
  if (gsel < 0) {
    if (tid == 0) a.out_ids[c.row] = NS_ERR_INVALID_DISTRIBUTION;
    return true;
  }
  if (warp != gsel / c.tpw) return true;
  // this warp copies its tile again and scans it in id order
  const int t = gsel % c.tpw;
  const bool pe = m->g_bin != 0;
  const unsigned long long tbefore = m->g_tbefore;
  const int sidx = seq % kWStages;
  if (lane == 0) issue_tile(c, warp, t, sidx, policy);
  if (!__all_sync(kFull, mbar_wait_bounded(c.sbar(warp, sidx), uint32_t(seq / kWStages) & 1u))) {
    if (lane == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
    return true;
  }
  uint8_t* st = c.stage(warp, sidx);
  float* F = reinterpret_cast<float*>(c.cx);  // the tile's values in column order (keys are dead)
  const int len = c.tile_len(warp, t), lead = c.tile_lead(warp, t);
  const int n_groups = (lead + len + VE - 1) / VE;
  const int base = warp * c.pw + t * TE;
  for (int q = lane; q < n_groups; q += 32) {
    float x[VE];
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int e = q * VE + i;
      if (e >= lead && e < lead + len) F[e - lead] = c.neg ? -x[i] : x[i];
    }
  }
  __syncwarp();
  patch_tile(c, warp, t, st, [&](bool has, float xp, int col) {  // history columns: penalised values
    if (has) F[col - base] = xp;
  });
  __syncwarp();
  auto mass_of = [&](int i) -> unsigned long long {
    const float x = F[i];
    if (!(x > -INFINITY)) return 0ull;
    const int b = wide_bin(x, M, r, S);
    if (b > jb || (b == jb && key_of(x, base + i) < keyL)) return 0ull;
    return wfx(yof(x));
  };
  const int per = (len + 31) / 32;
  const int i0 = min(lane * per, len), i1 = min(i0 + per, len);
  unsigned long long lm = 0;
  for (int i = i0; i < i1; ++i) lm += mass_of(i);
  unsigned long long ex = lm;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(kFull, ex, o);
    if (lane >= o) ex += v;
  }
  ex -= lm;
  unsigned long long cum = tbefore + ex;
  int pick = -1, last = -1;
  for (int i = i0; i < i1; ++i) {
    const unsigned long long e = mass_of(i);
    if (e == 0) continue;
    last = i;
    if (pick < 0 && !pe && cum + e > tgt) pick = i;
    cum += e;
  }
  const unsigned pm = __ballot_sync(kFull, pick >= 0);
  int col = -1;
  if (pm) {
    col = __shfl_sync(kFull, pick, __ffs(pm) - 1);
  } else {
    const unsigned lmk = __ballot_sync(kFull, last >= 0);
    if (lmk) col = __shfl_sync(kFull, last, 31 - __clz(lmk));
  }
  if (lane == 0)
    a.out_ids[c.row] = (col >= 0) ? int64_t(c.c0 + base + col) + a.vocab_offset : int64_t(NS_ERR_INVALID_DISTRIBUTION);
  return true;
}

template <int DT>
__device__ bool nucleus_wide(Ctx<DT>& c, const KArgs& a, int& seq, uint64_t policy, float topp) {
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float M = m->nuc_M;
  const double Z = m->nuc_Z;
  const float r = __frcp_rn(c.Tabs);
  uint32_t* h = m->hist;
  float* hm = reinterpret_cast<float*>(c.tacc);  // masses per bin (float: they only choose the bin)
  uint64_t* keys = reinterpret_cast<uint64_t*>(c.cx);
  auto key_of = [&](float x, int col) {
    const float y = __fdiv_rn(x, c.Tabs) + 0.0f;  // -0 and +0 tie
    return (uint64_t(f2key(y)) << 32) | uint64_t(~uint32_t(c.c0 + col));
  };
  const float dk = __fsub_rn(M, m->nuc_yk);  // +inf when unknown
  float D = fminf(dk + 4.5f, kWideMaxNats);
  float S = 0.0f;
  int jb = INT_MAX, nb = 0, n = 0, kb = 0, jg = INT_MAX, ng = 0;
  bool keyless = false;  // the window already counts more values than the keys hold
  bool exact = false;    // this attempt sums masses per bin (else guaranteed lower bounds)
  const float cov = m->nuc_cov;
  if (cov >= 0.0f && cov < 0.5f * topp) {  // the candidates hold little of the nucleus: it is far wider
    D = fminf(2.0f * D, kWideMaxNats);
    exact = true;
  }
  for (int att = 0; att < 6; ++att) {
    S = float(kWideBins - 1) / D;
    kb = (att == 0) ? int(fminf((dk + 3.5f) * S, float(kWideBins - 1))) : kWideBins - 1;  // NaN: all
    if (keyless) kb = 0;
    h[tid] = 0u;
    hm[tid] = 0.0f;
    if (tid == 0) {
      m->w_bin = INT_MAX;
      m->w_binb = INT_MAX;
      m->w_n = 0;
    }
    __syncthreads();
    warp_pass(
        c, seq, 0, policy, c.rep, c.pres, c.freq,
        [&](float x, int col) {
          if (x > -INFINITY) {
            const int b = wide_bin(x, M, r, S);
            if (b < kWideBins - 1) {
              atomicAdd(&h[b], 1u);
              if (exact) atomicAdd(&hm[b], __expf(__fmul_rn(x, r) - M));
              if (b < kb) {
                const int i = atomicAdd(&m->w_n, 1);
                if (i < kWideCap) keys[i] = key_of(x, col);
              }
            }
          }
        },
        [&](int) {}, wide_floor(M, D, c.Tabs));
    __syncthreads();
    if (m->flags & F_TIMEOUT) {  // every warp waited for its copies in flight
      if (tid == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
      return true;
    }
    n = m->w_n;
    // The bin where the cumulative mass first exceeds (p + 1e-6) Z by the
    // guaranteed lower bounds, or, with summed masses, (p + 2e-6) Z -- the
    // keys' prefix, which the float64 check then confirms -- and p Z, the
    // large-nucleus cut (whose pass recomputes the masses exactly and falls
    // back when the bin was not the right one).
    const int cnt = (tid < kWideBins - 1) ? int(h[tid]) : 0;
    const double lm = exact ? double(hm[tid < kWideBins - 1 ? tid : 0]) * (tid < kWideBins - 1 ? 1.0 : 0.0)
                            : double(cnt) * double(expf(-(float(tid) + 1.0f) * (D / float(kWideBins - 1)) - 1e-4f));
    double il = lm;
    int ic = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double vl = __shfl_up_sync(kFull, il, o);
      const int vc = __shfl_up_sync(kFull, ic, o);
      if (lane >= o) {
        il += vl;
        ic += vc;
      }
    }
    if (lane == 31) {
      m->d_red[warp] = il;
      m->i_red[warp] = ic;
    }
    __syncthreads();
    for (int w = 0; w < warp; ++w) {  // never reads the last warp's entries
      il += m->d_red[w];
      ic += m->i_red[w];
    }
    const double tk = (double(topp) + (exact ? 2e-6 : 1e-6)) * Z;
    if (il > tk && il - lm <= tk) {  // one thread at most
      m->w_bin = tid;
      m->i_red[kWarps - 1] = ic;
    }
    if (exact) {
      const double tg = double(topp) * Z;
      if (il > tg && il - lm <= tg) {
        m->w_binb = tid;
        m->w_cntb = cnt;
      }
    }
    if (tid == kThreads - 1) m->w_tot = ic;  // values counted in the window
    __syncthreads();
    jb = m->w_bin;
    nb = (jb != INT_MAX) ? m->i_red[kWarps - 1] : 0;
    jg = m->w_binb;
    ng = (jg != INT_MAX) ? m->w_cntb : 0;
    const int tot = m->w_tot;
    __syncthreads();
    if (jb != INT_MAX && nb <= kWideCap) break;  // the keys' prefix
    if (exact && (jg != INT_MAX || D >= kWideMaxNats)) break;
    keyless = keyless || tot > kWideCap;         // any prefix reaching the target is larger still
    if (jb == INT_MAX && D < kWideMaxNats) D = fminf(2.0f * D, kWideMaxNats);  // too little mass: wider
    exact = true;                                // later attempts sum masses per bin
  }
  if (jb == INT_MAX || nb == 0 || nb > kWideCap) {  // no keys' prefix: the large-nucleus path
    if (!exact || jg == INT_MAX || ng == 0 || ng > kWideCap) return false;
    return nucleus_big(c, a, seq, policy, topp, M, Z, r, S, jg);
  }
  if (jb >= kb || n > kWideCap) {  // the prefix lies past the keys' bins, or they overflowed
    if (tid == 0) m->w_n = 0;
    __syncthreads();
    warp_pass(
        c, seq, 0, policy, c.rep, c.pres, c.freq,
        [&](float x, int col) {
          if (x > -INFINITY && wide_bin(x, M, r, S) <= jb) {
            const int i = atomicAdd(&m->w_n, 1);
            if (i < kWideCap) keys[i] = key_of(x, col);
          }
        },
        [&](int) {}, wide_floor(M, float(jb + 1) / S, c.Tabs));
    __syncthreads();
    if (m->flags & F_TIMEOUT) {
      if (tid == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
      return true;
    }
    n = m->w_n;
    if (n > kWideCap || n == 0) return false;
  }
  uint64_t* tmp = reinterpret_cast<uint64_t*>(c.stages + size_t(kMergeCap) * 8);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff) + kRankMax;
  const float Sb = float(kBins - 1) / D;  // sort buckets: a function of y alone, so ties share one
  bucket_sort(
      m, keys, n, tmp, sorted,
      [&](uint64_t k) {
        const float d = (M - key2f(uint32_t(k >> 32))) * Sb;
        return d < float(kBins - 1) ? int(fmaxf(d, 0.0f)) : kBins - 1;
      },
      [](uint64_t x, uint64_t y) { return x > y; });
  // exact mass of the keys above the smallest scaled value
  {
    const uint32_t ylast = uint32_t(sorted[n - 1] >> 32);
    double cm = 0.0;
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t yk = uint32_t(sorted[i] >> 32);
      if (yk > ylast) cm += double(expf(__fsub_rn(key2f(yk), M)));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) cm += __shfl_xor_sync(kFull, cm, o);
    if (lane == 0) m->d_red[warp] = cm;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) tot += m->d_red[w];
    __syncthreads();
    if (!(tot > (double(topp) + 1e-6) * Z) || key2f(uint32_t(sorted[0] >> 32)) != M) return false;
  }
  c.K = n;  // no top-k: every key is a survivor
  finalize_keys(c, a, c.row, topp, sorted, n, n, Z);
  return true;
}

// ---------------------------------------------------------------------------
// Rows with kWideKFrom <= top_k <= kWideCap (one CTA per row).  The stream kept
// the kNucleusK largest values (with ties): the first is the row's largest
// scaled value M, the last sets the window scale dk.  One more pass counts the
// values within D = dk + 4 nats of M in 255 bins (d = M - x / |T| through a
// reciprocal; deeper values and their 16-byte groups skipped) and collects
// them as keys; the first bin where the count reaches k bounds the top-k (a
// window with fewer values is widened, twice as wide, up to 32 nats).  If the
// window holds more than kWideCap values, one more pass collects the bins up
// to that one (and the next, when they fit).  The keys are sorted; when the
// run of values tied with the k-th ends inside them, the finalise keeps the
// top-k with ties and applies top-p over them (reference sampler.py:116-131).
// Returns false (the same on every thread) when the row continues on the
// multi-pass path.
// ---------------------------------------------------------------------------
template <int DT>
__device__ bool wide_topk(Ctx<DT>& c, const KArgs& a, int& seq, uint64_t policy, int k, float topp) {
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float M = m->nuc_M;
  if (!(M > -INFINITY && M < INFINITY)) return false;  // the candidates did not give it
  const float r = __frcp_rn(c.Tabs);
  uint32_t* h = m->hist;
  uint64_t* keys = reinterpret_cast<uint64_t*>(c.cx);
  auto key_of = [&](float x, int col) {
    const float y = __fdiv_rn(x, c.Tabs) + 0.0f;  // -0 and +0 tie
    return (uint64_t(f2key(y)) << 32) | uint64_t(~uint32_t(c.c0 + col));
  };
  float D = fminf(__fsub_rn(M, m->nuc_yk) + 4.0f, kWideMaxNats);  // unknown scale: the widest
  float S = 0.0f;
  int jk = INT_MAX, nk = 0, n = 0;
  for (int att = 0; att < 4; ++att) {
    S = float(kWideBins - 1) / D;
    h[tid] = 0u;
    if (tid == 0) {
      m->w_bin = INT_MAX;
      m->w_n = 0;
    }
    __syncthreads();
    warp_pass(
        c, seq, 0, policy, c.rep, c.pres, c.freq,
        [&](float x, int col) {
          if (x > -INFINITY) {
            const int b = wide_bin(x, M, r, S);
            if (b < kWideBins - 1) {
              atomicAdd(&h[b], 1u);
              const int i = atomicAdd(&m->w_n, 1);
              if (i < kWideCap) keys[i] = key_of(x, col);
            }
          }
        },
        [&](int) {}, wide_floor(M, D, c.Tabs));
    __syncthreads();
    if (m->flags & F_TIMEOUT) {  // every warp waited for its copies in flight
      if (tid == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
      return true;
    }
    n = m->w_n;
    // the first bin where the count reaches k
    const int cnt = (tid < kWideBins - 1) ? int(h[tid]) : 0;
    int ic = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(kFull, ic, o);
      if (lane >= o) ic += v;
    }
    if (lane == 31) m->i_red[warp] = ic;
    __syncthreads();
    for (int w = 0; w < warp; ++w) ic += m->i_red[w];  // never reads the last warp's entry
    if (ic >= k && ic - cnt < k) {  // one thread at most
      m->w_bin = tid;
      m->i_red[kWarps - 1] = ic;
    }
    __syncthreads();
    jk = m->w_bin;
    nk = (jk != INT_MAX) ? m->i_red[kWarps - 1] : 0;
    __syncthreads();
    if (jk != INT_MAX || D >= kWideMaxNats) break;
    D = fminf(2.0f * D, kWideMaxNats);
  }
  if (jk == INT_MAX || nk > kWideCap) return false;
  int jc = kWideBins - 2;  // the last bin the keys hold
  if (n > kWideCap) {  // more values than keys: the bins up to jk (and the next if they fit)
    const int jp = (jk + 1 < kWideBins - 1 && nk + int(h[jk + 1]) <= kWideCap) ? jk + 1 : jk;
    jc = jp;
    if (tid == 0) m->w_n = 0;
    __syncthreads();
    warp_pass(
        c, seq, 0, policy, c.rep, c.pres, c.freq,
        [&](float x, int col) {
          if (x > -INFINITY && wide_bin(x, M, r, S) <= jp) {
            const int i = atomicAdd(&m->w_n, 1);
            if (i < kWideCap) keys[i] = key_of(x, col);
          }
        },
        [&](int) {}, wide_floor(M, float(jp + 1) / S, c.Tabs));
    __syncthreads();
    if (m->flags & F_TIMEOUT) {
      if (tid == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
      return true;
    }
    n = m->w_n;
    if (n > kWideCap || n < k) return false;
  }
  uint64_t* tmp = reinterpret_cast<uint64_t*>(c.stages + size_t(kMergeCap) * 8);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff) + kRankMax;
  const float Sb = float(kBins - 1) / D;  // sort buckets: a function of y alone, so ties share one
  bucket_sort(
      m, keys, n, tmp, sorted,
      [&](uint64_t kk) {
        const float d = (M - key2f(uint32_t(kk >> 32))) * Sb;
        return d < float(kBins - 1) ? int(fmaxf(d, 0.0f)) : kBins - 1;
      },
      [](uint64_t x, uint64_t y) { return x > y; });
  // the keys are an upper set of x: the run tied with the k-th is complete
  // when a smaller value follows it among them, or when its whole float
  // class lies in the bins the keys hold
  if (warp == 0) {
    const int nf = topk_with_ties(sorted, n, k);
    if (lane == 0) {
      int blo = 0, bhi = 0;
      const bool whole = nf < n || (y_class_bins(key2f(uint32_t(sorted[n - 1] >> 32)), c.Tabs, M, r, S, &blo, &bhi) &&
                                    bhi <= jc);
      m->w_L = whole ? nf : -1;
    }
  }
  __syncthreads();
  if (m->w_L < 0) return false;
  c.K = k;
  finalize_keys(c, a, c.row, topp, sorted, n, n);
  return true;
}

template <int DT>
__device__ void general_row(const Ctx<DT>& c, const KArgs& a, cg::cluster_group& cl, int CL, int rank, int& seq,
                            int pre_issued, uint64_t policy, float rep, float pres, float freq, float topp) {
  constexpr int VE = Ctx<DT>::VE, TE = Ctx<DT>::TE;
  Misc* m = c.m;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n_tiles_all = kWarps * c.tpw;
  unsigned long long* gh = reinterpret_cast<unsigned long long*>(c.cx);  // kGBins bins (candidate region)
  unsigned long long* tmass = reinterpret_cast<unsigned long long*>(c.tacc);
  int* tties = reinterpret_cast<int*>(tmass + n_tiles_all);
  const bool bigk = c.K > 0 && int64_t(c.K) < a.vocab_total;
  const bool usep = topp > 0.0f && topp < 1.0f;
  // Flags that decide control flow mid-way are only those no later pass can
  // set (a timeout may be set by a CTA that is already one pass ahead), so
  // every CTA takes the same branches; timeouts are checked once, in a window
  // where no CTA streams.
  const int hard = F_NAN | F_BADID | F_HIST;
  auto clear_gh = [&]() {
    for (int i = tid; i < kGBins; i += kThreads) gh[i] = 0;
  };
  auto cluster_flags = [&]() {
    int f = 0;
    for (int r = 0; r < CL; ++r) f |= cl.map_shared_rank(m, r)->flags;
    return f;
  };
  auto fail = [&](int status) {
    if (rank == 0 && tid == 0) a.out_ids[c.row] = status;
  };

  // ---- P1 ----
  clear_gh();
  if (tid == 0) m->g_maxk = 0u;
  __syncthreads();
  {
    float lmax = -INFINITY;
    bool bad = false;
    warp_pass(
        c, seq, pre_issued, policy, rep, pres, freq,
        [&](float x, int) {
          if (x != x || x == INFINITY) {
            bad = true;
          } else if (x > -INFINITY) {
            lmax = fmaxf(lmax, x);
            if (bigk) atomicAdd(&gh[f2key(x) >> 21], 1ull);
          }
        },
        [&](int) {});
    if (bad) atomicOr(&m->flags, F_NAN);
    if (lmax > -INFINITY) atomicMax(&m->g_maxk, f2key(lmax));
  }
  __syncthreads();
  cl.sync();
  const int fl = cluster_flags();
  unsigned maxk = 0;
  for (int r = 0; r < CL; ++r) maxk = max(maxk, cl.map_shared_rank(m, r)->g_maxk);
  if (fl & hard) {
    cl.sync();
    fail(status_from_flags(fl, false));
    return;
  }
  if (maxk == 0u) {  // no finite value: the reference's softmax is all-NaN
    cl.sync();
    fail(NS_ERR_INVALID_DISTRIBUTION);
    return;
  }
  const float M = __fdiv_rn(key2f(maxk), c.Tabs);
  if (!(M < INFINITY)) {
    cl.sync();
    fail(NS_ERR_INVALID_DISTRIBUTION);
    return;
  }

  // ---- P2, P3: the K-th largest x ----
  float lo = -INFINITY;
  if (bigk) {
    cluster_digit(cl, CL, m, gh, kGBins, (unsigned long long)c.K, false);
    int d0 = m->g_bin;
    unsigned long long krem = (unsigned long long)c.K - m->g_before;
    cl.sync();
    if (d0 >= 0) {
      clear_gh();
      __syncthreads();
      warp_pass(
          c, seq, 0, policy, rep, pres, freq,
          [&](float x, int) {
            const uint32_t k = f2key(x);
            if (x > -INFINITY && x == x && (k >> 21) == uint32_t(d0)) atomicAdd(&gh[(k >> 10) & 0x7FFu], 1ull);
          },
          [&](int) {}, key2f(uint32_t(d0) << 21));
      __syncthreads();
      cl.sync();
      cluster_digit(cl, CL, m, gh, kGBins, krem, false);
      const int d1 = m->g_bin;
      krem -= m->g_before;
      cl.sync();
      clear_gh();
      __syncthreads();
      const uint32_t pre = (uint32_t(d0) << 11) | uint32_t(d1);
      warp_pass(
          c, seq, 0, policy, rep, pres, freq,
          [&](float x, int) {
            const uint32_t k = f2key(x);
            if (x > -INFINITY && x == x && (k >> 10) == pre) atomicAdd(&gh[k & 0x3FFu], 1ull);
          },
          [&](int) {}, key2f(pre << 10));
      __syncthreads();
      cl.sync();
      cluster_digit(cl, CL, m, gh, 1024, krem, false);
      const uint32_t kth = (pre << 10) | uint32_t(m->g_bin);
      lo = scaled_lower_bound(key2f(kth), c.Tabs);
      cl.sync();
    }
  }

  // ---- P4: masses of the top-k survivors ----
  auto surv = [&](float x) { return x >= lo && x > -INFINITY; };
  clear_gh();
  __syncthreads();
  {
    unsigned long long acc = 0;
    warp_pass(
        c, seq, 0, policy, rep, pres, freq,
        [&](float x, int) {
          if (!surv(x)) return;
          const float y = __fdiv_rn(x, c.Tabs);
          const unsigned long long e = to_fx(expf(__fsub_rn(y, M)));
          acc += e;
          if (usep) atomicAdd(&gh[f2key(y + 0.0f) >> 21], e);
        },
        [&](int t) {
          const unsigned long long sum = warp_sum_u64(acc);
          acc = 0;
          if (lane == 0) tmass[warp * c.tpw + t] = sum;
        },
        lo);
  }
  __syncthreads();
  if (tid == 0) {
    unsigned long long z = 0;
    for (int w = 0; w < kWarps; ++w)
      for (int t = 0; t < c.wtiles(w); ++t) z += tmass[w * c.tpw + t];
    m->g_mass = z;
  }
  __syncthreads();
  cl.sync();
  unsigned long long Z = 0;
  for (int r = 0; r < CL; ++r) Z += cl.map_shared_rank(m, r)->g_mass;

  // ---- P5, P6, P7: the top-p cut ----
  bool cut = false;
  float cval = 0.0f;
  unsigned long long n_keep = 0, ecut = 0;
  if (usep) {
    const unsigned long long target0 = (unsigned long long)(double(topp) * double(Z));
    cluster_digit(cl, CL, m, gh, kGBins, target0, true);
    const int b0 = m->g_bin;
    unsigned long long O = m->g_before;
    cl.sync();
    if (b0 >= 0) {
      cut = true;
      clear_gh();
      __syncthreads();
      warp_pass(
          c, seq, 0, policy, rep, pres, freq,
          [&](float x, int) {
            if (!surv(x)) return;
            const float y = __fdiv_rn(x, c.Tabs);
            const uint32_t k = f2key(y + 0.0f);
            if ((k >> 21) == uint32_t(b0)) atomicAdd(&gh[(k >> 10) & 0x7FFu], to_fx(expf(__fsub_rn(y, M))));
          },
          [&](int) {}, fmaxf(lo, x_floor_of_y(key2f(uint32_t(b0) << 21), c.Tabs)));
      __syncthreads();
      cl.sync();
      cluster_digit(cl, CL, m, gh, kGBins, target0 - O, true);
      const int b1 = m->g_bin;
      O += m->g_before;
      cl.sync();
      clear_gh();
      __syncthreads();
      const uint32_t pre = (uint32_t(b0) << 11) | uint32_t(b1);
      warp_pass(
          c, seq, 0, policy, rep, pres, freq,
          [&](float x, int) {
            if (!surv(x)) return;
            const float y = __fdiv_rn(x, c.Tabs);
            const uint32_t k = f2key(y + 0.0f);
            if ((k >> 10) == pre) atomicAdd(&gh[k & 0x3FFu], to_fx(expf(__fsub_rn(y, M))));
          },
          [&](int) {}, fmaxf(lo, x_floor_of_y(key2f(pre << 10), c.Tabs)));
      __syncthreads();
      cl.sync();
      cluster_digit(cl, CL, m, gh, 1024, target0 - O, true);
      const int b2 = m->g_bin;
      O += m->g_before;
      cval = key2f((pre << 10) | uint32_t(b2));
      ecut = to_fx(expf(__fsub_rn(cval, M)));
      unsigned long long binmass = 0;
      for (int r = 0; r < CL; ++r) binmass += cl.map_shared_rank(gh, r)[b2];
      const unsigned long long n_c = ecut ? binmass / ecut : 0;
      n_keep = ecut ? min(n_c, (target0 - O) / ecut + 1) : n_c;
      cl.sync();
      // P7: mass above the cut and ties at it, per tile
      {
        unsigned long long acc = 0;
        int ties = 0;
        warp_pass(
            c, seq, 0, policy, rep, pres, freq,
            [&](float x, int) {
              if (!surv(x)) return;
              const float y = __fdiv_rn(x, c.Tabs) + 0.0f;
              if (y > cval)
                acc += to_fx(expf(__fsub_rn(y, M)));
              else if (y == cval)
                ++ties;
            },
            [&](int t) {
              const unsigned long long sum = warp_sum_u64(acc);
              const int tt = __reduce_add_sync(kFull, unsigned(ties));
              acc = 0;
              ties = 0;
              if (lane == 0) {
                tmass[warp * c.tpw + t] = sum;
                tties[warp * c.tpw + t] = tt;
              }
            },
            fmaxf(lo, x_floor_of_y(cval, c.Tabs)));
      }
      __syncthreads();
      if (tid == 0) {
        int tsum = 0;
        for (int w = 0; w < kWarps; ++w)
          for (int t = 0; t < c.wtiles(w); ++t) tsum += tties[w * c.tpw + t];
        m->g_ties = tsum;
      }
      __syncthreads();
      cl.sync();
      unsigned long long tb = 0;  // ties in the CTAs before this one (column order)
      for (int r = 0; r < rank; ++r) tb += (unsigned long long)cl.map_shared_rank(m, r)->g_ties;
      if (tid == 0) {  // kept mass per tile: above the cut + the first n_keep ties in id order
        unsigned long long z = 0;
        for (int w = 0; w < kWarps; ++w)
          for (int t = 0; t < c.wtiles(w); ++t) {
            const int gt = w * c.tpw + t;
            const unsigned long long nt = (unsigned long long)tties[gt];
            const unsigned long long kept = (n_keep > tb) ? min(nt, n_keep - tb) : 0ull;
            tmass[gt] += kept * ecut;
            tties[gt] = int(tb);  // ties before this tile, for P8
            tb += nt;
            z += tmass[gt];
          }
        m->g_mass = z;
      }
      __syncthreads();
      cl.sync();
    }
  }
  // ---- inverse CDF: CTA, tile, then P8 inside the tile ----
  const bool timed_out = (cluster_flags() & F_TIMEOUT) != 0;
  unsigned long long ZS = 0;
  for (int r = 0; r < CL; ++r) ZS += cl.map_shared_rank(m, r)->g_mass;
  const float u = a.uniforms ? c.u_pre : philox_uniform(a.seed, a.offset, uint64_t(c.row));
  const unsigned long long target = (unsigned long long)(double(u) * double(ZS));
  int rsel = -1, rlast = -1;
  unsigned long long rbefore = 0, run = 0;
  for (int r = 0; r < CL; ++r) {
    const unsigned long long mr = cl.map_shared_rank(m, r)->g_mass;
    if (mr > 0) rlast = r;
    if (rsel < 0 && run + mr > target) {
      rsel = r;
      rbefore = run;
    }
    run += mr;
  }
  bool past_end = false;
  if (rsel < 0) {  // u * total at or beyond the last step: the last kept value
    rsel = rlast;
    past_end = true;
  }
  cl.sync();  // nobody reads remote shared memory past this point
  if (timed_out) {
    fail(NS_ERR_DEVICE_TIMEOUT);
    return;
  }
  if (rank != rsel) return;
  if (tid == 0) {
    int tsel = -1, tlast = -1;
    unsigned long long tbefore = rbefore, tr = rbefore;
    for (int w = 0; w < kWarps; ++w)
      for (int t = 0; t < c.wtiles(w); ++t) {
        const int gt = w * c.tpw + t;
        if (tmass[gt] > 0) tlast = gt;
        if (tsel < 0 && !past_end && tr + tmass[gt] > target) {
          tsel = gt;
          tbefore = tr;
        }
        tr += tmass[gt];
      }
    if (tsel < 0) {
      tsel = tlast;
      past_end = true;
    }
    m->g_tile = tsel;
    m->g_tbefore = tbefore;
    m->g_bin = past_end ? 1 : 0;
  }
  __syncthreads();
  const int gsel = m->g_tile;
  if (gsel < 0 || warp != gsel / c.tpw) return;
  // P8: this warp reloads its tile and scans it in id order
  const int t = gsel % c.tpw;
  const bool pe = m->g_bin != 0;
  const unsigned long long tbefore = m->g_tbefore;
  const int sidx = seq % kWStages;
  if (lane == 0) issue_tile(c, warp, t, sidx, policy);
  if (!__all_sync(kFull, mbar_wait_bounded(c.sbar(warp, sidx), uint32_t(seq / kWStages) & 1u))) {
    if (lane == 0) a.out_ids[c.row] = NS_ERR_DEVICE_TIMEOUT;
    return;
  }
  uint8_t* st = c.stage(warp, sidx);
  float* F = reinterpret_cast<float*>(c.cx);  // fp32 values of the tile in column order
  const int len = c.tile_len(warp, t), lead = c.tile_lead(warp, t);
  const int n_groups = (lead + len + VE - 1) / VE;
  const int base = warp * c.pw + t * TE;

  for (int q = lane; q < n_groups; q += 32) {
    float x[VE];
    unpack16<DT>(*reinterpret_cast<const uint4*>(st + q * 16), x);
#pragma unroll
    for (int i = 0; i < VE; ++i) {
      const int e = q * VE + i;
      if (e >= lead && e < lead + len) F[e - lead] = c.neg ? -x[i] : x[i];
    }
  }
  __syncwarp();
  // history columns get their penalised values on top of the raw ones
  patch_tile(c, warp, t, st, [&](bool has, float xp, int col) {
    if (has) F[col - base] = xp;
  });
  __syncwarp();
  const unsigned long long ties_before = cut ? (unsigned long long)tties[gsel] : 0ull;
  auto mass_of = [&](float x, bool& tie) {
    tie = false;
    if (!surv(x)) return 0ull;
    const float y = __fdiv_rn(x, c.Tabs) + 0.0f;
    if (cut) {
      if (y < cval) return 0ull;
      if (y == cval) {
        tie = true;
        return ecut;
      }
    }
    return to_fx(expf(__fsub_rn(y, M)));
  };
  const int per = (len + 31) / 32;
  const int i0 = min(lane * per, len), i1 = min(i0 + per, len);
  unsigned long long lm = 0;
  int lt = 0;
  for (int i = i0; i < i1; ++i) {
    bool tie;
    const unsigned long long e = mass_of(F[i], tie);
    if (tie) {
      ++lt;
    } else {
      lm += e;
    }
  }
  int lt_ex = lt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, lt_ex, o);
    if (lane >= o) lt_ex += v;
  }
  lt_ex -= lt;
  // kept ties of this lane's chunk are those with global tie rank < n_keep
  unsigned long long rank0 = ties_before + (unsigned long long)lt_ex;
  unsigned long long kept_here = 0;
  if (cut && lt > 0 && n_keep > rank0) kept_here = min((unsigned long long)lt, n_keep - rank0);
  lm += kept_here * ecut;
  unsigned long long lm_ex = lm;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(kFull, lm_ex, o);
    if (lane >= o) lm_ex += v;
  }
  lm_ex -= lm;
  unsigned long long cum = tbefore + lm_ex, trank = rank0;
  int pick = -1, last = -1;
  for (int i = i0; i < i1; ++i) {
    bool tie;
    unsigned long long e = mass_of(F[i], tie);
    if (tie) {
      e = (trank < n_keep) ? ecut : 0ull;
      ++trank;
    }
    if (e == 0) continue;
    last = i;
    if (pick < 0 && !pe && cum + e > target) pick = i;
    cum += e;
  }
  // the first lane holding the crossing wins; past the end: the last kept value
  const unsigned pm = __ballot_sync(kFull, pick >= 0);
  int col = -1;
  if (pm) {
    col = __shfl_sync(kFull, pick, __ffs(pm) - 1);
  } else {
    const unsigned lmk = __ballot_sync(kFull, last >= 0);
    if (lmk) col = __shfl_sync(kFull, last, 31 - __clz(lmk));
  }
  if (lane == 0)
    a.out_ids[c.row] = (col >= 0) ? int64_t(c.c0 + base + col) + a.vocab_offset : int64_t(NS_ERR_INVALID_DISTRIBUTION);
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(kThreads, 2) sample_kernel(const __grid_constant__ KArgs a) {
  using C_ = Ctx<DT>;
  extern __shared__ __align__(128) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  const int64_t row = blockIdx.x / CL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  C_ c;
  c.stages = smem;
  c.bar = reinterpret_cast<uint64_t*>(smem + a.off_bar);
  c.cx = reinterpret_cast<float*>(smem + a.off_cand);
  c.cid = reinterpret_cast<int*>(smem + a.off_cand + kWarps * kCapW * 4);
  c.bits = reinterpret_cast<uint32_t*>(smem + a.off_bits);
  c.pre = reinterpret_cast<uint16_t*>(smem + a.off_pre);
  c.cnt = reinterpret_cast<int*>(smem + a.off_cnt);
  c.colr = reinterpret_cast<int*>(smem + a.off_colr);
  c.pval = reinterpret_cast<float*>(smem + a.off_pval);
  c.nwords = a.nwords;
  c.tacc = smem + a.off_tacc;
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
  else if (topk >= kWideKFrom && int64_t(topk) < a.vocab_total && topk <= kWideCap && CL == 1 && !a.vp_keys)
    mode = MODE_WIDEK;
  else if (topk > 0 && int64_t(topk) < a.vocab_total && topk <= kFastK)
    mode = MODE_FAST;
  else if (!(topk > 0 && int64_t(topk) < a.vocab_total) && !a.vp_keys && !(topp > 0.0f && topp < 1.0f))
    mode = MODE_SOFTMAX;
  else if (!(topk > 0 && int64_t(topk) < a.vocab_total) && !a.vp_keys)
    mode = MODE_NUCLEUS;
  else
    mode = MODE_GENERAL;
  // NUCLEUS (top-k off, top-p on): the FAST filter keeps the kNucleusK largest
  // with ties as candidates, and the tile masses give the row's total; when the
  // candidates hold more than p of it the cut lies among them
  const bool fastlike = (mode == MODE_FAST || mode == MODE_NUCLEUS || mode == MODE_WIDEK);
  if (a.vp_keys && mode == MODE_GENERAL) {  // no candidate record for these rows
    if (rank == 0 && tid == 0) a.out_ids[row] = NS_ERR_UNSUPPORTED;
    return;
  }
  c.neg = T < 0.0f;
  c.Tabs = fabsf(T);
  c.K = (mode == MODE_NUCLEUS || mode == MODE_WIDEK) ? kNucleusK : topk;
  int64_t h0 = 0, h1 = 0;
  if (a.hist_offsets) {
    h0 = a.hist_offsets[row];
    h1 = a.hist_offsets[row + 1];
  }
  const bool pen = (h1 > h0) && (rep != 1.0f || pres != 0.0f || freq != 0.0f);
  c.pen = pen;
  c.rep = rep;
  c.pres = pres;
  c.freq = freq;
  c.u_pre = a.uniforms ? a.uniforms[row] : 0.0f;
  // The first kHB * kThreads history ids are loaded before any tile copy is
  // queued, and stay in registers for both prologue passes.
  constexpr int kHB = 8;
  int ids0[kHB];
  unsigned ids0_ok = 0;
  if (pen) {
#pragma unroll
    for (int q = 0; q < kHB; ++q) {
      const int64_t i = h0 + int64_t(q) * kThreads + tid;
      ids0[q] = (i < h1) ? a.hist_ids[i] : 0;
      ids0_ok |= (i < h1 ? 1u : 0u) << q;
    }
  }
  c.rowp = reinterpret_cast<const uint8_t*>(a.logits) + size_t(row) * size_t(a.row_stride) * C_::ES;
  c.row = row;
  c.c0 = int(min(int64_t(rank) * a.per_cta, a.vocab));
  c.c1 = int(min(int64_t(c.c0) + a.per_cta, a.vocab));
  c.pw = a.per_warp;
  c.tpw = a.tpw;

  if (tid == 0) {
    for (int s = 0; s < kWarps * kWStages; ++s) mbar_init(&c.bar[s], 1);
    fence_mbar_init();
    m->flags = 0;
    m->n_merge = 0;
    m->choose = INT_MAX;
    m->g_best = -INFINITY;
    m->g_idx = INT_MAX;
    m->hist_g = 0;
    for (int w = 0; w < kWarps; ++w) m->pub[w] = 0u;
  }
  if (pen) {
    for (int i = tid; i < a.nwords; i += kThreads) c.bits[i] = 0u;
    for (int i = tid; i < a.cnt_cap; i += kThreads) c.cnt[i] = 0;
  }
  __syncthreads();

  const uint64_t policy = l2_policy_evict_first();
  const bool streams = (mode != MODE_GENERAL);  // GENERAL rows stream in general_row()
  // each warp starts its first copies now so they overlap the history prologue
  if (lane == 0) {
    const int nt = c.wtiles(warp);
    for (int t = 0; t < min(kWStages, nt); ++t) issue_tile(c, warp, t, t, policy);
  }

  // ---- history: membership bitmap, ranks and occurrence counts ----
  // Fire-and-forget shared atomics only: bits are set with atomicOr; each warp
  // scans the popcounts of its own columns' words (16-bit prefixes, the warp
  // totals in segoff), which gives every distinct id a rank in column order;
  // the counts are accumulated with atomicAdd at that rank.  The penalised
  // values are computed when their tiles land (patch_tile).
  if (pen) {
#pragma unroll
    for (int q = 0; q < kHB; ++q) {
      if ((ids0_ok >> q) & 1u) {
        const int id = ids0[q];
        const int64_t lc = int64_t(id) - a.vocab_offset;
        if (id < 0 || int64_t(id) >= a.vocab_total) {
          atomicOr(&m->flags, F_BADID);
        } else if (lc >= c.c0 && lc < c.c1) {
          const int rel = int(lc - c.c0);
          atomicOr(&c.bits[rel >> 5], 1u << (rel & 31));
        }
      }
    }
    auto for_more_ids = [&](auto f) {  // ids past the first kHB * kThreads
      for (int64_t base = h0 + int64_t(kThreads) * kHB; base < h1; base += int64_t(kThreads) * kHB) {
        int ids[kHB];
#pragma unroll
        for (int q = 0; q < kHB; ++q) {
          const int64_t i = base + int64_t(q) * kThreads + tid;
          ids[q] = (i < h1) ? a.hist_ids[i] : 0;
        }
#pragma unroll
        for (int q = 0; q < kHB; ++q)
          if (base + int64_t(q) * kThreads + tid < h1) f(ids[q]);
      }
    };
    for_more_ids([&](int id) {
      if (id < 0 || int64_t(id) >= a.vocab_total) {
        atomicOr(&m->flags, F_BADID);
        return;
      }
      const int64_t lc = int64_t(id) - a.vocab_offset;
      if (lc >= c.c0 && lc < c.c1) {
        const int rel = int(lc - c.c0);
        atomicOr(&c.bits[rel >> 5], 1u << (rel & 31));
      }
    });
    __syncthreads();
    {  // this warp's words: 4 per lane per step, 16-byte loads
      const int wpw = c.pw >> 5;  // a multiple of 4
      const uint32_t* wb = c.bits + warp * wpw;
      uint16_t* wp = c.pre + warp * wpw;
      uint32_t run = 0;
      for (int j0 = 0; j0 < wpw; j0 += 128) {
        const int j = j0 + 4 * lane;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (j < wpw) v = *reinterpret_cast<const uint4*>(wb + j);
        const uint32_t p0 = __popc(v.x), p1 = __popc(v.y), p2 = __popc(v.z), p3 = __popc(v.w);
        const uint32_t sum = p0 + p1 + p2 + p3;
        uint32_t incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t u = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += u;
        }
        const uint32_t e0 = run + incl - sum;
        if (j < wpw) {
          const uint32_t e1 = e0 + p0, e2 = e1 + p1, e3 = e2 + p2;
          *reinterpret_cast<uint2*>(wp + j) = make_uint2((e0 & 0xFFFFu) | (e1 << 16), (e2 & 0xFFFFu) | (e3 << 16));
        }
        run += __shfl_sync(kFull, incl, 31);
      }
      if (lane == 0) m->i_red[warp] = int(run);
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0;
      bool wide = false;
      for (int w = 0; w < kWarps; ++w) {
        m->segoff[w] = acc;
        acc += m->i_red[w];
        wide |= m->i_red[w] > 0xFFFF;  // the 16-bit prefixes would wrap
      }
      m->segoff[kWarps] = acc;
      if (wide) {
        atomicOr(&m->flags, F_HIST);
      } else if (acc > a.cnt_cap) {
        if (a.hist_ws && acc <= a.hist_ws_cap)
          m->hist_g = 1;
        else
          atomicOr(&m->flags, F_HIST);
      }
    }
    __syncthreads();
    if (m->hist_g && !(m->flags & F_HIST)) {  // this CTA's rank arrays in its workspace slot
      int32_t* base = a.hist_ws + size_t(blockIdx.x) * 3 * size_t(a.hist_ws_cap);
      c.cnt = base;
      c.colr = base + a.hist_ws_cap;
      c.pval = reinterpret_cast<float*>(base + 2 * size_t(a.hist_ws_cap));
      for (int i = tid; i < m->segoff[kWarps]; i += kThreads) c.cnt[i] = 0;
      __syncthreads();
    }
    if (!(m->flags & F_HIST)) {
      const int wpw = c.pw >> 5;
      auto count = [&](int rel) {
        const int wi = rel >> 5, b = rel & 31;
        const int r = m->segoff[wi / wpw] + c.pre[wi] + __popc(c.bits[wi] & ((1u << b) - 1u));
        atomicAdd(&c.cnt[r], 1);
        c.colr[r] = rel;
      };
#pragma unroll
      for (int q = 0; q < kHB; ++q)
        if ((ids0_ok >> q) & 1u) {
          const int64_t lc = int64_t(ids0[q]) - a.vocab_offset;
          if (ids0[q] >= 0 && lc >= c.c0 && lc < c.c1) count(int(lc - c.c0));
        }
      for_more_ids([&](int id) {
        const int64_t lc = int64_t(id) - a.vocab_offset;
        if (id >= 0 && lc >= c.c0 && lc < c.c1) count(int(lc - c.c0));
      });
    }
    __syncthreads();
    // without ranks nothing may be patched (the row reports F_HIST)
    if (m->flags & F_HIST) c.pen = false;
  }

  // ---- stream: every warp independently ----
  WarpCand s;
  s.x = c.cx + warp * kCapW;
  s.col = c.cid + warp * kCapW;
  s.tau = -INFINITY;
  s.n = 0;
  s.ovf = false;
  float best = -INFINITY;
  int bidx = INT_MAX;
  int n_ready = 0;
  if (fastlike) {
    // Seed: each warp publishes the kq-th largest of its 32 lane maxima over
    // its first kWStages tiles (distinct elements); after one block barrier
    // every warp starts from the shared bound.
    float tmax = -INFINITY;
    const int nr = min(kWStages, c.wtiles(warp));
    bool ready = true;
    for (int t = 0; t < nr; ++t) ready = ready && __all_sync(kFull, mbar_wait_bounded(c.sbar(warp, t), 0u));
    if (ready) {
      n_ready = nr;
      for (int t = 0; t < nr; ++t) {
        uint8_t* st = c.stage(warp, t);
        if (c.pen) {
          mask_tile(c, warp, t, st);
          __syncwarp();
        }
        tmax = fmaxf(tmax, c.neg ? tile_lane_max<DT, true>(c, warp, t, st) : tile_lane_max<DT, false>(c, warp, t, st));
      }
    }
    publish_key(c, warp_kth_lanes(tmax > -INFINITY ? f2key(tmax) : 0u, share_kq(c.K)));
    __syncthreads();
    read_shared_tau(c, s);
  }
  bool ok = true;
  if (streams) ok = stream_warp(c, mode, policy, 0, n_ready, s, best, bidx);
  // this warp's penalised history values: the rank range of its columns
  if (ok && c.pen) {
    penalize_segment(c, warp);
    const int hr0 = m->segoff[warp], hr1 = m->segoff[warp + 1];
    if (mode == MODE_GREEDY) {
      for (int r = hr0 + lane; r < hr1; r += 32) {
        const float x = c.pval[r];
        const int col = c.c0 + c.colr[r];
        if (better(x, col, best, bidx)) {
          best = x;
          bidx = col;
        }
      }
    } else if (fastlike && !s.ovf) {
      for (int r0 = hr0; r0 < hr1; r0 += 32) {
        const int r = r0 + lane;
        const bool has = r < hr1;
        fast_emit(c, s, has, has ? c.pval[r] : 0.0f, has ? c.colr[r] : 0);
      }
    }
  }
  if (fastlike && s.ovf && lane == 0) atomicOr(&m->flags, F_OVF);
  if (mode == MODE_SOFTMAX) {
    softmax_tail(c, a, policy, cluster, CL, rank);
    return;
  }
  int seq_next = c.wtiles(warp);  // copies this warp has made
  if (mode != MODE_GENERAL) {
    if (row_tail(c, a, cluster, CL, rank, mode, ok, s, best, bidx, topp)) return;
    __syncthreads();  // the row continues below
    if (mode == MODE_NUCLEUS && CL == 1 && nucleus_wide(c, a, seq_next, policy, topp)) return;
    if (mode == MODE_WIDEK && wide_topk(c, a, seq_next, policy, topk, topp)) return;
  }
  if (fastlike) {  // every warp's final bound; survivors of the tightest
    if (ok) publish_bound(c, s);
    __syncthreads();
    if (!s.ovf) {
      read_shared_tau(c, s);
      warp_drop_below(s);
    }
  }
  if (mode == MODE_GREEDY) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(kFull, best, o);
      const int oi = __shfl_xor_sync(kFull, bidx, o);
      if (better(ob, oi, best, bidx)) {
        best = ob;
        bidx = oi;
      }
    }
  }
  if (lane == 0) {
    m->wn[warp] = (fastlike && ok && !s.ovf) ? s.n : 0;
    m->wbest[warp] = best;
    m->widx[warp] = bidx;
  }
  __syncthreads();
  if (tid == 0 && mode == MODE_GREEDY) {
    float b = m->wbest[0];
    int bi = m->widx[0];
    for (int w = 1; w < kWarps; ++w)
      if (better(m->wbest[w], m->widx[w], b, bi)) {
        b = m->wbest[w];
        bi = m->widx[w];
      }
    m->g_best = b;
    m->g_idx = bi;
  }
  __syncthreads();

  // ---- cluster merge ----
  cluster.sync();
  {
    // GENERAL rows, and FAST rows whose ties overflowed a buffer anywhere in
    // the cluster, continue with the multi-pass path (a cluster-uniform
    // decision: every CTA reads every CTA's flags).
    int fl_all = 0;
    for (int r = 0; r < CL; ++r) fl_all |= cluster.map_shared_rank(m, r)->flags;
    const bool hard = (fl_all & (F_NAN | F_TIMEOUT | F_BADID | F_HIST)) != 0;
    if (a.vp_keys && mode == MODE_FAST && (fl_all & F_OVF) && !hard) {
      cluster.sync();  // every CTA has read the others' flags
      if (rank == 0 && tid == 0) a.out_ids[row] = NS_ERR_CANDIDATE_OVERFLOW;
      return;
    }
    if (mode == MODE_GENERAL || (fastlike && (fl_all & F_OVF) && !hard)) {
      cluster.sync();
      c.K = topk;  // NUCLEUS rows filtered with kNucleusK
      if (tid == 0) m->flags &= ~F_OVF;
      __syncthreads();
      int seq = (mode == MODE_GENERAL) ? 0 : seq_next;
      const int pre = (mode == MODE_GENERAL) ? min(kWStages, c.wtiles(warp)) : 0;
      general_row(c, a, cluster, CL, rank, seq, pre, policy, rep, pres, freq, topp);
      return;
    }
  }
  if (rank == 0) {
    if (tid == 0) {
      int fl = 0, tot = 0;
      float b = -INFINITY;
      int bi = INT_MAX;
      for (int r = 0; r < CL; ++r) {
        Misc* rm = cluster.map_shared_rank(m, r);
        fl |= rm->flags;
        m->rc0[r] = int(min(int64_t(r) * a.per_cta, a.vocab));
        for (int w = 0; w < kWarps; ++w) {
          m->roff[r * kWarps + w] = tot;
          tot += rm->wn[w];
        }
        if (better(rm->g_best, rm->g_idx, b, bi)) {
          b = rm->g_best;
          bi = rm->g_idx;
        }
      }
      m->roff[CL * kWarps] = tot;
      m->flags = fl;
      if (mode == MODE_GREEDY) {
        const int st = status_from_flags(fl, true);
        if (st != NS_OK) {
          a.out_ids[row] = int64_t(st);
        } else if (a.vp_keys) {  // one key; NaN sorts above every value
          const uint32_t hi = (b != b) ? 0xFFFFFFFFu : f2key(b + 0.0f);
          const uint32_t gid = uint32_t(int64_t(bi) + a.vocab_offset);
          a.vp_keys[row * a.vp_cap] = int64_t((uint64_t(hi) << 32) | uint64_t(~gid));
          a.out_ids[row] = 1;
        } else {
          a.out_ids[row] = int64_t(bi) + a.vocab_offset;
        }
      } else if (status_from_flags(fl, false) != NS_OK) {
        a.out_ids[row] = status_from_flags(fl, false);
      }
    }
    __syncthreads();
    if (mode == MODE_FAST && status_from_flags(m->flags, false) == NS_OK) {
      if (m->roff[CL * kWarps] <= kRankMax) {
        gather_keys(c, cluster, CL);
      } else if (a.vp_keys) {
        if (tid == 0) a.out_ids[row] = NS_ERR_CANDIDATE_OVERFLOW;
      } else {
        leader_gather(c, a, cluster, CL);
      }
    }
  }
  cluster.sync();
  if (rank == 0 && mode == MODE_FAST && status_from_flags(m->flags, false) == NS_OK) {
    if (m->roff[CL * kWarps] <= kRankMax)
      rank_finalize(c, a, row, topp, m->roff[CL * kWarps]);
    else if (!a.vp_keys)
      finalize_row(c, a, row, topp);
  }
}

// ---------------------------------------------------------------------------
// vocab-parallel merge: one CTA per row over the all-gathered records of
// n_ranks column slices.  Record of rank r (int64): [batch] counts or
// statuses, then [batch][cap] keys (f2key(y) << 32 | ~global id).  Every
// element of the row's global top-k (with ties at the k-th scaled value)
// lies in its own slice's top-k with ties, so the union holds the global set
// and the result equals the single-device call on the whole row.
// ---------------------------------------------------------------------------

constexpr int kMaxPeers = 8;  // ranks of a peer-memory exchange (one NVLink domain)

struct VpMerge {
  const int64_t* rec;                // n_ranks consecutive records, or null:
  const int64_t* peer[kMaxPeers];    // ... rank r's record read in place (peer memory)
  const int64_t* flags;              // null, or this rank's flags: wait for flags[r] >= *epoch
  const int64_t* epoch;              // this rank's step counter (set by vp_signal_kernel)
  int n_ranks;
  int cap;
  int64_t batch;
};

struct VpSignal {
  int64_t* flags[kMaxPeers];  // rank r's flag array (peer memory for r != me)
  int64_t* epoch;             // this rank's step counter (device memory)
  int n_ranks;
  int me;
};

// After this rank's local step (the previous kernel on the stream): the step
// counter advances and every rank's flags[me] = the new count, released at
// system scope.  The count lives in device memory so that a captured CUDA
// graph advances it on every replay.
__global__ void vp_signal_kernel(const __grid_constant__ VpSignal s) {
  const int r = threadIdx.x;
  int64_t e = 0;
  if (r == 0) {
    e = *s.epoch + 1;
    *s.epoch = e;
  }
  e = __shfl_sync(0xFFFFFFFFu, e, 0);
  __threadfence_system();
  if (r < s.n_ranks) st_release_sys(s.flags[r] + s.me, e);
}

__device__ __forceinline__ int status_rank(int64_t st) {  // single-device priority order
  switch (int(st)) {
    case NS_ERR_DEVICE_TIMEOUT: return 0;
    case NS_ERR_TOKEN_ID_OUT_OF_RANGE: return 1;
    case NS_ERR_HISTORY_TOO_LONG: return 2;
    case NS_ERR_UNSUPPORTED: return 3;
    case NS_ERR_INVALID_DISTRIBUTION: return 4;
    case NS_ERR_CANDIDATE_OVERFLOW: return 5;
    default: return 6;
  }
}

__global__ void __launch_bounds__(kThreads) vp_merge_kernel(const __grid_constant__ KArgs a,
                                                            const __grid_constant__ VpMerge v) {
  using C_ = Ctx<NS_DTYPE_F32>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  C_ c;
  c.stages = smem;
  c.m = reinterpret_cast<Misc*>(smem + kStageBytes);
  c.row = row;
  const float T = a.temperature[row];
  const int topk = a.top_k[row];
  const float topp = a.top_p[row];
  c.K = topk;
  c.Tabs = fabsf(T);
  c.neg = T < 0.0f;
  c.u_pre = a.uniforms ? a.uniforms[row] : 0.0f;
  Misc* m = c.m;
  const int64_t rlen = v.batch * (1 + int64_t(v.cap));
  auto record = [&](int r) { return v.rec ? v.rec + r * rlen : v.peer[r]; };
  if (v.flags) {  // peer records: wait (bounded) until every rank has signalled this step
    if (tid == 0) m->r_digit = 0;
    __syncthreads();
    if (tid < v.n_ranks && !flag_wait_bounded(v.flags + tid, *v.epoch)) atomicOr(&m->r_digit, 1);
    __syncthreads();
    if (m->r_digit) {
      if (tid == 0) a.out_ids[row] = NS_ERR_DEVICE_TIMEOUT;
      return;
    }
  }
  if (tid == 0) {
    int64_t err = 0;
    int tot = 0;
    for (int r = 0; r < v.n_ranks; ++r) {
      const int64_t h = record(r)[row];
      m->roff[r] = tot;
      if (h < 0) {
        if (err == 0 || status_rank(h) < status_rank(err)) err = h;
      } else {
        tot += int(h < int64_t(v.cap) ? h : int64_t(v.cap));
      }
    }
    m->roff[v.n_ranks] = tot;
    m->flags = int(err);
  }
  __syncthreads();
  if (m->flags != 0) {
    if (tid == 0) a.out_ids[row] = m->flags;
    return;
  }
  if (T == 0.0f) {  // greedy: the largest key over the ranks
    if (warp == 0) {
      uint64_t best = 0;
      for (int r = lane; r < v.n_ranks; r += 32) {
        const int64_t* base = record(r);
        if (base[row] > 0) best = max(best, uint64_t(base[v.batch + row * v.cap]));
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(kFull, best, o));
      if (lane == 0) a.out_ids[row] = best ? int64_t(~uint32_t(best)) : NS_ERR_INVALID_DISTRIBUTION;
    }
    return;
  }
  if (!(topk > 0 && int64_t(topk) < a.vocab_total && topk <= kFastK)) {
    if (tid == 0) a.out_ids[row] = NS_ERR_UNSUPPORTED;
    return;
  }
  // Each rank's keys arrive sorted (descending) and distinct across ranks, so a
  // key's position in the union is its index in its own list plus, for every
  // other list, the number of keys above it.  The lists are staged in shared
  // memory; keys placed past kRankMax cannot be among the kept ones unless a
  // tie run reaches them (finalize_keys reports that as overflow).
  const int n = m->roff[v.n_ranks];
  if (n > kMergeStage) {
    if (tid == 0) a.out_ids[row] = NS_ERR_CANDIDATE_OVERFLOW;
    return;
  }
  uint64_t* lists = reinterpret_cast<uint64_t*>(c.stages);
  uint64_t* sorted = reinterpret_cast<uint64_t*>(c.stages + kRankKeysOff) + kRankMax;
  for (int r = warp; r < v.n_ranks; r += kWarps) {
    const int cnt = m->roff[r + 1] - m->roff[r];
    const int64_t* src = record(r) + v.batch + row * v.cap;
    for (int i = lane; i < cnt; i += 32) lists[m->roff[r] + i] = uint64_t(src[i]);
  }
  __syncthreads();
  place_sorted_lists(lists, m->roff, v.n_ranks, n, sorted);
  finalize_keys(c, a, row, topp, sorted, min(n, kRankMax), n);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Layout {
  uint32_t off_bar, off_cand, off_bits, off_pre, off_cnt, off_colr, off_pval, off_tacc, off_misc, total;
};

static uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

static Layout make_layout(int nwords, int cnt_cap, int n_tiles_all) {
  Layout L;
  uint32_t o = kStageBytes;
  L.off_bar = o;
  o += kWarps * kWStages * 8;
  o = align_up(o, 16);
  // FAST candidate buffers / GENERAL histograms / tile expansion; during the
  // history prologue (before any of those) the same bytes hold the bitmap,
  // 16-byte aligned so every warp's words start on 16 bytes.
  L.off_cand = o;
  L.off_bits = o;
  o += std::max<uint32_t>(uint32_t(kCandBytes), uint32_t(nwords) * 4);
  o = align_up(o, 16);
  L.off_pre = o;
  o += uint32_t(nwords) * 2;
  o = align_up(o, 16);
  L.off_cnt = o;
  o += uint32_t(cnt_cap) * 4;
  L.off_colr = o;
  o += uint32_t(cnt_cap) * 4;
  L.off_pval = o;
  o += uint32_t(cnt_cap) * 4;
  o = align_up(o, 16);
  L.off_tacc = o;  // GENERAL: per-(warp, tile) mass (fixed point) and tie count; wide NUCLEUS: bin masses
  o += std::max<uint32_t>(uint32_t(n_tiles_all) * 12, uint32_t(kWideBins) * 8);
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

static int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NS_ERR_CUDA;
  DeviceInfo* di = &g_dev[dev];
  std::lock_guard<std::mutex> lk(g_mu);
  if (di->sms == 0) {
    int sms = 0, optin = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return NS_ERR_CUDA;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
      return NS_ERR_CUDA;
    di->max_smem_optin = optin;
    di->sms = sms;
  }
  *out = di;
  return NS_OK;
}

// Launch shape of a call: CTAs per row (a cluster) and the columns of a CTA
// and of a warp.
struct Geom {
  int CL;
  int64_t per, pw, span;
};

template <int DT>
static Geom geometry(int64_t batch, int64_t V, int sms) {
  using C_ = Ctx<DT>;
  Geom g;
  // CTAs per row: enough rows x CTAs to cover the SMs, each warp >= 1 tile.
  g.CL = 1;
  while (g.CL < kMaxCluster && batch * g.CL < sms && V / (2 * g.CL) >= int64_t(kWarps) * C_::TE) g.CL *= 2;
  g.per = (V + g.CL - 1) / g.CL;
  g.per = (g.per + C_::VE - 1) / C_::VE * C_::VE;
  g.pw = (g.per + kWarps - 1) / kWarps;
  g.pw = (g.pw + 127) / 128 * 128;  // warp ranges start on 16-byte groups of bitmap words
  g.span = int64_t(kWarps) * g.pw;  // columns one CTA may own
  return g;
}

// Distinct history ids a CTA may meet, and the workspace bytes for the rank
// arrays of every CTA when that is more than shared memory holds (else 0).
static int64_t hist_cap(int64_t max_history, const Geom& g) {
  return std::min<int64_t>(std::max<int64_t>(max_history, 1), g.span);
}
static size_t hist_ws_need(int64_t batch, int64_t max_history, const Geom& g) {
  const int64_t cap = hist_cap(max_history, g);
  return cap > kHistSmem ? size_t(batch) * size_t(g.CL) * 12 * size_t(cap) : 0;
}

template <int DT>
static int launch(const KArgs& base, int64_t batch, ns_stream_t stream) {
  using C_ = Ctx<DT>;
  DeviceInfo* di = nullptr;
  if (const int rc = device_info(&di)) return rc;
  KArgs a = base;
  const Geom g = geometry<DT>(batch, a.vocab, di->sms);
  const int CL = g.CL;
  a.per_cta = int(g.per);
  a.per_warp = int(g.pw);
  a.tpw = int((g.pw + C_::TE - 1) / C_::TE);
  const int n_tiles_all = kWarps * a.tpw;
  a.nwords = a.hist_ids ? int((g.span + 31) / 32) : 0;
  a.cnt_cap = a.hist_ids ? int(std::min<int64_t>(hist_cap(a.max_history, g), kHistSmem)) : 0;
  a.hist_ws = nullptr;
  a.hist_ws_cap = 0;
  if (a.hist_ids) {
    const size_t need = hist_ws_need(batch, a.max_history, g);
    if (need > 0) {
      if (!a.ws || a.ws_bytes < need || (reinterpret_cast<uintptr_t>(a.ws) & 255u) != 0)
        return NS_ERR_WORKSPACE_TOO_SMALL;
      a.hist_ws = static_cast<int32_t*>(a.ws);
      a.hist_ws_cap = int(hist_cap(a.max_history, g));
    }
  }
  const Layout L = make_layout(a.nwords, a.cnt_cap, n_tiles_all);
  a.merge_cap = kMergeCap;
  a.off_bar = L.off_bar;
  a.off_cand = L.off_cand;
  a.off_bits = L.off_bits;
  a.off_pre = L.off_pre;
  a.off_cnt = L.off_cnt;
  a.off_colr = L.off_colr;
  a.off_pval = L.off_pval;
  a.off_tacc = L.off_tacc;
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

static int vp_merge_launch(const KArgs& a, const VpMerge& v, ns_stream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NS_ERR_CUDA;
  const size_t smem_bytes = kStageBytes + sizeof(Misc);
  {
    static bool configured[64] = {};
    std::lock_guard<std::mutex> lk(g_mu);
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(vp_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem_bytes)) !=
          cudaSuccess)
        return NS_ERR_CUDA;
      configured[dev] = true;
    }
  }
  vp_merge_kernel<<<unsigned(v.batch), kThreads, smem_bytes, reinterpret_cast<cudaStream_t>(stream)>>>(a, v);
  if (cudaGetLastError() != cudaSuccess) return NS_ERR_CUDA;
  return NS_OK;
}


// ---------------------------------------------------------------------------
// debug readback: the penalised logits of whole rows
// ---------------------------------------------------------------------------
// One block per row.  The row is widened to fp32 into out; then every history
// position counts the occurrences of its id in the row's history (chunks of
// the ids staged in shared memory) and the first occurrence of each distinct
// id writes penalize(x, count) -- the same device function, hence the same
// bits, as the sampling kernels.  O(H^2 / threads) per row: a checking tool,
// not a hot path.
constexpr int kPenChunk = 4096;

template <int DT>
__global__ void __launch_bounds__(kThreads) penalize_rows_kernel(const __grid_constant__ KArgs a, float* out,
                                                                 int64_t out_stride, int32_t* row_status) {
  using E = Elem<DT>;
  __shared__ int ids_s[kPenChunk];
  __shared__ int bad;
  const int64_t row = blockIdx.x;
  const typename E::raw* src = reinterpret_cast<const typename E::raw*>(a.logits) + row * a.row_stride;
  float* dst = out + row * out_stride;
  for (int64_t j = threadIdx.x; j < a.vocab; j += kThreads) dst[j] = E::widen(src[j]);
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  const float rep = a.rep ? a.rep[row] : 1.0f;
  const float pres = a.pres ? a.pres[row] : 0.0f;
  const float freq = a.freq ? a.freq[row] : 0.0f;
  const int64_t h0 = a.hist_offsets ? a.hist_offsets[row] : 0, h1 = a.hist_offsets ? a.hist_offsets[row + 1] : 0;
  const bool active = (rep != 1.0f || pres != 0.0f || freq != 0.0f) && h1 > h0;
  if (active) {
    for (int64_t i = h0 + threadIdx.x; i < h1; i += kThreads) {
      const int id = a.hist_ids[i];
      if (id < 0 || int64_t(id) >= a.vocab) atomicOr(&bad, 1);
    }
  }
  __syncthreads();
  if (bad) {
    if (threadIdx.x == 0) row_status[row] = NS_ERR_TOKEN_ID_OUT_OF_RANGE;
    return;
  }
  if (active) {
    const int64_t n = h1 - h0;
    for (int64_t mine0 = 0; mine0 < n; mine0 += kThreads) {  // every thread takes part in the staging
      const int64_t mi = mine0 + threadIdx.x;
      const int my = (mi < n) ? a.hist_ids[h0 + mi] : -1;
      int cnt = 0;
      bool first = true;
      for (int64_t c0 = 0; c0 < n; c0 += kPenChunk) {
        const int cn = int((n - c0 < int64_t(kPenChunk)) ? (n - c0) : int64_t(kPenChunk));
        __syncthreads();
        for (int k = threadIdx.x; k < cn; k += kThreads) ids_s[k] = a.hist_ids[h0 + c0 + k];
        __syncthreads();
        if (mi < n) {
          for (int k = 0; k < cn; ++k) {
            const bool eq = ids_s[k] == my;
            cnt += eq ? 1 : 0;
            if (eq && c0 + k < mi) first = false;
          }
        }
      }
      if (mi < n && first) dst[my] = penalize(E::widen(src[my]), cnt, rep, pres, freq);
    }
  }
  if (threadIdx.x == 0) row_status[row] = NS_OK;
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
  if (vocab > (int64_t(1) << 24) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
  *out_bytes = 0;
  if (max_history <= ns::kHistSmem) return NS_OK;
  // The launch shape depends on the device's SM count; without a device the
  // widest clusters the vocabulary allows bound it (the bytes never shrink
  // as clusters widen).
  ns::DeviceInfo* di = nullptr;
  const int sms = ns::device_info(&di) == NS_OK ? di->sms : INT_MAX;
  if (!di) (void)cudaGetLastError();
  const size_t f32 = ns::hist_ws_need(batch, max_history, ns::geometry<NS_DTYPE_F32>(batch, vocab, sms));
  const size_t b16 = ns::hist_ws_need(batch, max_history, ns::geometry<NS_DTYPE_BF16>(batch, vocab, sms));
  *out_bytes = std::max(f32, b16);
  return NS_OK;
}

int ns_sampler_smem_bytes(int dtype, int64_t batch, int64_t vocab, int64_t max_history, int sm_count,
                          size_t* out_bytes) {
  if (!out_bytes || batch <= 0 || vocab <= 0 || max_history < 0 || sm_count <= 0) return NS_ERR_INVALID_ARGUMENT;
  if (vocab > (int64_t(1) << 24) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
  if (dtype != NS_DTYPE_F32 && dtype != NS_DTYPE_BF16 && dtype != NS_DTYPE_F16) return NS_ERR_UNSUPPORTED_DTYPE;
  // the arithmetic of launch(): geometry, then the shared-memory layout of a
  // row with a history (the bitmap, prefixes and rank arrays present)
  auto size = [&](auto geom, int te) {
    const ns::Geom g = geom;
    const int64_t tpw = (g.pw + te - 1) / te;
    const int nwords = max_history > 0 ? int((g.span + 31) / 32) : 0;
    const int cnt_cap = max_history > 0 ? int(std::min<int64_t>(ns::hist_cap(max_history, g), ns::kHistSmem)) : 0;
    return size_t(ns::make_layout(nwords, cnt_cap, int(ns::kWarps * tpw)).total);
  };
  if (dtype == NS_DTYPE_F32)
    *out_bytes = size(ns::geometry<NS_DTYPE_F32>(batch, vocab, sm_count), ns::Ctx<NS_DTYPE_F32>::TE);
  else if (dtype == NS_DTYPE_BF16)
    *out_bytes = size(ns::geometry<NS_DTYPE_BF16>(batch, vocab, sm_count), ns::Ctx<NS_DTYPE_BF16>::TE);
  else
    *out_bytes = size(ns::geometry<NS_DTYPE_F16>(batch, vocab, sm_count), ns::Ctx<NS_DTYPE_F16>::TE);
  return NS_OK;
}

int ns_sample(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
              const int32_t* hist_ids, const int64_t* hist_offsets, int64_t max_history,
              const float* temperature, const int32_t* top_k, const float* top_p,
              const float* repetition_penalty, const float* presence_penalty, const float* frequency_penalty,
              const float* uniforms, uint64_t philox_seed, uint64_t philox_offset, int64_t* out_ids,
              void* workspace, size_t workspace_bytes, ns_stream_t stream) {
  if (dtype != NS_DTYPE_F32 && dtype != NS_DTYPE_BF16 && dtype != NS_DTYPE_F16) return NS_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || vocab <= 0 || row_stride < vocab || max_history < 0) return NS_ERR_INVALID_ARGUMENT;
  if (vocab > (int64_t(1) << 24) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
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
  a.max_history = max_history;
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
  a.ws = workspace;
  a.ws_bytes = workspace_bytes;
  switch (dtype) {
    case NS_DTYPE_F32: return ns::launch<NS_DTYPE_F32>(a, batch, stream);
    case NS_DTYPE_BF16: return ns::launch<NS_DTYPE_BF16>(a, batch, stream);
    default: return ns::launch<NS_DTYPE_F16>(a, batch, stream);
  }
}

int ns_penalize_debug(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                      const int32_t* hist_ids, const int64_t* hist_offsets, const float* repetition_penalty,
                      const float* presence_penalty, const float* frequency_penalty, float* out,
                      int64_t out_stride, int32_t* row_status, ns_stream_t stream) {
  if (dtype != NS_DTYPE_F32 && dtype != NS_DTYPE_BF16 && dtype != NS_DTYPE_F16) return NS_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || vocab <= 0 || row_stride < vocab || out_stride < vocab) return NS_ERR_INVALID_ARGUMENT;
  if (vocab > (int64_t(1) << 24) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
  if ((hist_ids == nullptr) != (hist_offsets == nullptr)) return NS_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NS_OK;
  if (!logits || !out || !row_status) return NS_ERR_INVALID_ARGUMENT;
  ns::KArgs a = {};
  a.logits = logits;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.hist_ids = hist_ids;
  a.hist_offsets = hist_offsets;
  a.rep = repetition_penalty;
  a.pres = presence_penalty;
  a.freq = frequency_penalty;
  const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case NS_DTYPE_F32:
      ns::penalize_rows_kernel<NS_DTYPE_F32><<<unsigned(batch), ns::kThreads, 0, s>>>(a, out, out_stride, row_status);
      break;
    case NS_DTYPE_BF16:
      ns::penalize_rows_kernel<NS_DTYPE_BF16><<<unsigned(batch), ns::kThreads, 0, s>>>(a, out, out_stride, row_status);
      break;
    default:
      ns::penalize_rows_kernel<NS_DTYPE_F16><<<unsigned(batch), ns::kThreads, 0, s>>>(a, out, out_stride, row_status);
  }
  return cudaGetLastError() == cudaSuccess ? NS_OK : NS_ERR_CUDA;
}

int ns_vp_record_int64s(int64_t batch, int cap, int64_t* out_count) {
  if (!out_count || batch < 0 || cap < 1 || cap > ns::kRankMax) return NS_ERR_INVALID_ARGUMENT;
  *out_count = batch * (1 + int64_t(cap));
  return NS_OK;
}

int ns_vp_local(const void* logits, int dtype, int64_t batch, int64_t vocab_local, int64_t row_stride,
                int64_t vocab_offset, int64_t vocab_total, const int32_t* hist_ids, const int64_t* hist_offsets,
                int64_t max_history, const float* temperature, const int32_t* top_k, const float* top_p,
                const float* repetition_penalty, const float* presence_penalty, const float* frequency_penalty,
                int cap, int64_t* record, void* workspace, size_t workspace_bytes, ns_stream_t stream) {
  if (dtype != NS_DTYPE_F32 && dtype != NS_DTYPE_BF16 && dtype != NS_DTYPE_F16) return NS_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || vocab_local <= 0 || row_stride < vocab_local || max_history < 0) return NS_ERR_INVALID_ARGUMENT;
  if (vocab_offset < 0 || vocab_total < vocab_offset + vocab_local || vocab_total > (int64_t(1) << 24) ||
      batch > (int64_t(1) << 24))
    return NS_ERR_INVALID_ARGUMENT;
  if (cap < 1 || cap > ns::kRankMax) return NS_ERR_INVALID_ARGUMENT;
  if ((hist_ids == nullptr) != (hist_offsets == nullptr)) return NS_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NS_OK;
  if (!logits || !temperature || !top_k || !top_p || !record) return NS_ERR_INVALID_ARGUMENT;
  ns::KArgs a = {};
  a.logits = logits;
  a.vocab = vocab_local;
  a.row_stride = row_stride;
  a.vocab_offset = vocab_offset;
  a.vocab_total = vocab_total;
  a.hist_ids = hist_ids;
  a.hist_offsets = hist_offsets;
  a.max_history = max_history;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.rep = repetition_penalty;
  a.pres = presence_penalty;
  a.freq = frequency_penalty;
  a.out_ids = record;           // [batch] counts / statuses
  a.vp_keys = record + batch;   // [batch][cap] keys
  a.vp_cap = cap;
  a.ws = workspace;
  a.ws_bytes = workspace_bytes;
  switch (dtype) {
    case NS_DTYPE_F32: return ns::launch<NS_DTYPE_F32>(a, batch, stream);
    case NS_DTYPE_BF16: return ns::launch<NS_DTYPE_BF16>(a, batch, stream);
    default: return ns::launch<NS_DTYPE_F16>(a, batch, stream);
  }
}

int ns_vp_merge(const int64_t* gathered, int n_ranks, int64_t batch, int cap, int64_t vocab_total,
                const float* temperature, const int32_t* top_k, const float* top_p, const float* uniforms,
                uint64_t philox_seed, uint64_t philox_offset, int64_t* out_ids, ns_stream_t stream) {
  if (n_ranks < 1 || n_ranks > ns::kMaxLists || batch < 0 || cap < 1 || cap > ns::kRankMax) return NS_ERR_INVALID_ARGUMENT;
  if (vocab_total <= 0 || vocab_total > (int64_t(1) << 24) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NS_OK;
  if (!gathered || !temperature || !top_k || !top_p || !out_ids) return NS_ERR_INVALID_ARGUMENT;
  ns::KArgs a = {};
  a.vocab = vocab_total;
  a.vocab_offset = 0;
  a.vocab_total = vocab_total;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.uniforms = uniforms;
  a.seed = philox_seed;
  a.offset = philox_offset;
  a.out_ids = out_ids;
  a.merge_cap = ns::kMergeCap;
  ns::VpMerge v = {};
  v.rec = gathered;
  v.n_ranks = n_ranks;
  v.cap = cap;
  v.batch = batch;
  return ns::vp_merge_launch(a, v, stream);
}

int ns_vp_merge_peers(const int64_t* const* rank_records, int n_ranks, const int64_t* my_flags,
                      const int64_t* epoch, int64_t batch, int cap, int64_t vocab_total, const float* temperature,
                      const int32_t* top_k, const float* top_p, const float* uniforms, uint64_t philox_seed,
                      uint64_t philox_offset, int64_t* out_ids, ns_stream_t stream) {
  if (n_ranks < 1 || n_ranks > ns::kMaxPeers || batch < 0 || cap < 1 || cap > ns::kRankMax || !epoch)
    return NS_ERR_INVALID_ARGUMENT;
  if (vocab_total <= 0 || vocab_total > (int64_t(1) << 24) || batch > (int64_t(1) << 24)) return NS_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NS_OK;
  if (!rank_records || !my_flags || !temperature || !top_k || !top_p || !out_ids) return NS_ERR_INVALID_ARGUMENT;
  ns::KArgs a = {};
  a.vocab = vocab_total;
  a.vocab_offset = 0;
  a.vocab_total = vocab_total;
  a.temperature = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.uniforms = uniforms;
  a.seed = philox_seed;
  a.offset = philox_offset;
  a.out_ids = out_ids;
  a.merge_cap = ns::kMergeCap;
  ns::VpMerge v = {};
  v.rec = nullptr;
  for (int r = 0; r < n_ranks; ++r) {
    if (!rank_records[r]) return NS_ERR_INVALID_ARGUMENT;
    v.peer[r] = rank_records[r];
  }
  v.flags = my_flags;
  v.epoch = epoch;
  v.n_ranks = n_ranks;
  v.cap = cap;
  v.batch = batch;
  return ns::vp_merge_launch(a, v, stream);
}

int ns_vp_signal(int64_t* const* rank_flags, int n_ranks, int my_rank, int64_t* epoch, ns_stream_t stream) {
  if (!rank_flags || n_ranks < 1 || n_ranks > ns::kMaxPeers || my_rank < 0 || my_rank >= n_ranks || !epoch)
    return NS_ERR_INVALID_ARGUMENT;
  ns::VpSignal sg = {};
  for (int r = 0; r < n_ranks; ++r) {
    if (!rank_flags[r]) return NS_ERR_INVALID_ARGUMENT;
    sg.flags[r] = rank_flags[r];
  }
  sg.n_ranks = n_ranks;
  sg.me = my_rank;
  sg.epoch = epoch;
  ns::vp_signal_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(sg);
  return cudaGetLastError() == cudaSuccess ? NS_OK : NS_ERR_CUDA;
}

int ns_vp_peer_alloc(size_t bytes, void** out_ptr) {
  if (!out_ptr || bytes == 0) return NS_ERR_INVALID_ARGUMENT;
  *out_ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return NS_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return NS_ERR_CUDA;
  }
  *out_ptr = p;
  return NS_OK;
}

int ns_vp_peer_free(void* ptr) {
  if (!ptr) return NS_OK;
  return cudaFree(ptr) == cudaSuccess ? NS_OK : NS_ERR_CUDA;
}

static_assert(sizeof(cudaIpcMemHandle_t) == NS_IPC_HANDLE_BYTES, "IPC handle size");

int ns_ipc_handle(const void* ptr, void* out_handle) {
  if (!ptr || !out_handle) return NS_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return NS_ERR_CUDA;
  std::memcpy(out_handle, &h, sizeof(h));
  return NS_OK;
}

int ns_ipc_open(const void* handle, void** out_ptr) {
  if (!handle || !out_ptr) return NS_ERR_INVALID_ARGUMENT;
  *out_ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return NS_ERR_CUDA;
  *out_ptr = p;
  return NS_OK;
}

int ns_ipc_close(void* ptr) {
  if (!ptr) return NS_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? NS_OK : NS_ERR_CUDA;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Device-resident histories: append one sampled id per row
// ---------------------------------------------------------------------------
// The reference rebuilds every row's history as prompt + outputs lists on the
// host each step (engine/context_builder.py:208-213, outputs appended at
// driver/output_processor.py:46).  Here the history CSR stays on the device:
// after a sampling step, row b's ids are copied to out at offset
// offsets[b] + b and the row's new id follows them, so out_offsets[b] =
// offsets[b] + b.  One CTA per row (grid-stride over rows beyond the grid);
// writes past out_capacity elements are dropped (a caller that sized out too
// small gets a truncated history, never a stray write).
namespace ns {

constexpr int kAppendThreads = 256;

__global__ void __launch_bounds__(kAppendThreads) hist_append_kernel(const int32_t* __restrict__ ids,
                                                                     const int64_t* __restrict__ offsets,
                                                                     int64_t batch, const int64_t* __restrict__ new_ids,
                                                                     int32_t* __restrict__ out_ids,
                                                                     int64_t* __restrict__ out_offsets,
                                                                     int64_t out_capacity) {
  for (int64_t b = blockIdx.x; b < batch; b += gridDim.x) {
    const int64_t h0 = offsets ? offsets[b] : 0, h1 = offsets ? offsets[b + 1] : 0;
    const int64_t dst = h0 + b;
    for (int64_t i = h0 + threadIdx.x; i < h1; i += kAppendThreads)
      if (i + b < out_capacity) out_ids[i + b] = ids[i];
    if (threadIdx.x == 0) {
      // an error status (negative) is stored as is: the next sampling step
      // reports NS_ERR_TOKEN_ID_OUT_OF_RANGE for that row
      const int64_t v = new_ids[b];
      const int32_t id = (v >= 0 && v <= INT32_MAX) ? int32_t(v) : int32_t(-1);
      if (dst + (h1 - h0) < out_capacity) out_ids[dst + (h1 - h0)] = id;
      out_offsets[b] = dst;
      if (b == batch - 1) out_offsets[batch] = h1 + batch;
    }
  }
}

}  // namespace ns

extern "C" int ns_hist_append(const int32_t* hist_ids, const int64_t* hist_offsets, int64_t batch,
                              const int64_t* new_ids, int32_t* out_hist_ids, int64_t* out_hist_offsets,
                              int64_t out_capacity, ns_stream_t stream) {
  if (batch < 0 || out_capacity < 0) return NS_ERR_INVALID_ARGUMENT;
  if ((hist_ids == nullptr) != (hist_offsets == nullptr)) return NS_ERR_INVALID_ARGUMENT;
  if (batch == 0) return NS_OK;
  if (!new_ids || !out_hist_ids || !out_hist_offsets || out_capacity < batch) return NS_ERR_INVALID_ARGUMENT;
  const unsigned grid = unsigned(std::min<int64_t>(batch, 65535));
  ns::hist_append_kernel<<<grid, ns::kAppendThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      hist_ids, hist_offsets, batch, new_ids, out_hist_ids, out_hist_offsets, out_capacity);
  return cudaGetLastError() == cudaSuccess ? NS_OK : NS_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// ns_sample without a caller workspace
// ---------------------------------------------------------------------------
// For callers that may not allocate device memory around a sampling step (an
// engine whose memory pool owns every byte, a plug-in inside a runtime that
// does all allocation).  The scratch ns_sample takes from its caller -- the
// long-history rank arrays -- lives instead in this fixed array, which the
// CUDA module holds on every device that loads it until the process exits.
// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory: the device address comes from cudaGetSymbolAddress, looked up once
// per device with that device current, on its first call.
namespace ns {

static __device__ __align__(256) unsigned char g_noalloc_scratch[NS_NOALLOC_SCRATCH_BYTES];

static void* g_noalloc_addr[64];

static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return NS_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
      (void)cudaGetLastError();
      return NS_ERR_CUDA;
    }
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return NS_OK;
}

}  // namespace ns

extern "C" {

int ns_sample_noalloc(const void* logits, int dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                      const int32_t* hist_ids, const int64_t* hist_offsets, int64_t max_history,
                      const float* temperature, const int32_t* top_k, const float* top_p,
                      const float* repetition_penalty, const float* presence_penalty,
                      const float* frequency_penalty, const float* uniforms, uint64_t philox_seed,
                      uint64_t philox_offset, int64_t* out_ids, ns_stream_t stream) {
  if (dtype != NS_DTYPE_F32 && dtype != NS_DTYPE_BF16 && dtype != NS_DTYPE_F16) return NS_ERR_UNSUPPORTED_DTYPE;
  if (batch < 0 || vocab <= 0 || row_stride < vocab || max_history < 0) return NS_ERR_INVALID_ARGUMENT;
  // the same sizing ns_sample checks a caller workspace against
  size_t need = 0;
  if (const int rc = ns_sampler_workspace_bytes(batch, vocab, hist_ids ? max_history : 0, &need)) return rc;
  if (need > NS_NOALLOC_SCRATCH_BYTES) return NS_ERR_WORKSPACE_TOO_SMALL;
  void* scratch = nullptr;
  if (const int rc = ns::noalloc_scratch(&scratch)) return rc;
  // The kernel zeroes the counts it accumulates in the scratch and writes the
  // column and value arrays before reading them, so nothing is cleared here.
  return ns_sample(logits, dtype, batch, vocab, row_stride, hist_ids, hist_offsets, max_history, temperature,
                   top_k, top_p, repetition_penalty, presence_penalty, frequency_penalty, uniforms, philox_seed,
                   philox_offset, out_ids, scratch, NS_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
