// B200 (sm_100a) batched token sampler: greedy / temperature / top-k / top-p with an
// inverse-CDF draw, one thread-block cluster per logits row, every row of a batch in one launch.
//
// Replaces pagedbatch/sampling.py:10-27 (sample_token), called per row by
// pagedbatch/engine.py:133-139. Exact semantics are stated in include/pagedbatch_b200.h.
//
// Per row (cluster of C CTAs, each owning a contiguous slice of the row):
//  1. Stream: the slice goes HBM -> shared memory through a ring of 1-D bulk copies (TMA engine,
//     mbarrier completion, no multicast). Each element becomes key = x / T (IEEE fp32); the CTA
//     keeps the max key (lowest index on ties) and, for top-k rows with k <= KSMALL, a candidate
//     list of keys >= a running threshold (the k-th largest key seen so far: a lower bound of the
//     row's k-th key, so no survivor is ever dropped).
//  2. Greedy rows finish here. Small top-k rows finish in rank 0's shared memory: exact k-th key
//     by bisection over the candidates of all C CTAs (copied through distributed shared memory),
//     the survivors sorted by (key desc, index asc), fixed-point weights scanned for the top-p
//     cut and the draw.
//  3. Other rows (temperature-only, top-p over the full vocabulary, large k): the cluster re-reads
//     its slices (L2) in histogram passes. Pass Z bins the fixed-point weight mass by distance to
//     the max; each selection (k-th key, top-p cut, draw) walks down from the bin holding its
//     target, either gathering the bin's elements into rank 0 for an exact finish or refining by
//     11-bit digits of the key; a tie group larger than the gather buffer is resolved by counting.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "../../include/pagedbatch_b200.h"
#include "pb_device.cuh"

namespace cg = cooperative_groups;
using namespace pb;

namespace {

constexpr int NT = 256;             // threads per CTA
constexpr int NW = NT / 32;
constexpr int CHUNK_BYTES = 32768;  // bytes per staged chunk (the ring holds two: a warp's fixed cost per
                                    // chunk, wait and release, is paid once per 32 KB)
constexpr int RING_BYTES = 65536;
constexpr int MAX_STAGE = 16;
constexpr int CAND_CAP = 4096;      // candidate entries per CTA
constexpr int SLOTS = CAND_CAP / NT; // candidate slots per thread
constexpr int CP_CHUNKS = 4;        // chunks between CTA checkpoints (128 KB; rows with a small top_k)
constexpr uint32_t BUCKET = 32;     // keys left between the bisection bounds when it stops early
constexpr int KSMALL = 1024;        // largest top_k resolved from the streamed candidates
constexpr int KCAP = 2048;          // survivors of the small path sorted in rank 0
constexpr int NBIN = 2048;          // histogram bins of the cooperative selection
constexpr int GCAP = 4096;          // elements gathered into rank 0 for an exact finish
constexpr int WAIT_POLLS = 20000;   // bounded mbarrier wait (~seconds) before a row reports a timeout
constexpr float MASS_RANGE = 27.75f;  // below max - 27.75 the 2^40-scaled weight is 0

static_assert(CAND_CAP % NT == 0, "slots split evenly");

// dynamic shared memory regions (bytes)
constexpr int REGION_A = RING_BYTES;  // ring | local histograms | small-path survivors
constexpr int REGION_B = 32768;  // candidates | gather list (rank 0)
constexpr int REGION_C = 0;
constexpr int DYN_SMEM = REGION_A + REGION_B + REGION_C;

struct Args {
  const char* logits;
  int64_t n_rows, vocab, row_stride;
  const int32_t* row_index;
  const pb_row_params* params;
  int64_t* out_token;
  pb_row_info* out_info;
  float* out_probs;
  const pb_row_info* only_fallback;  // if set: sample only the rows whose status there is PB_ROW_FALLBACK
  int32_t complement;    // skip the rows the streaming kernel settled (it ran first on the stream)
  uint8_t* cand_out;     // vocabulary-parallel shard mode: per-row candidate records (else null)
  int32_t cand_cap;      // entries per record
  int64_t vocab_offset;  // global index of this shard's first column
};

// one row's candidate record: header, then `count` composites (scaled key, global index)
__host__ __device__ constexpr int64_t record_bytes(int cap) { return (int64_t)sizeof(pb_cand_header) + 8 * (int64_t)cap; }

// decision record broadcast by rank 0 (read by peers through DSMEM)
struct Dec {
  uint32_t lo, hi;       // current key interval of the selection
  uint64_t above_w;      // weight strictly above the interval
  uint64_t above_c;      // count strictly above the interval
  uint64_t cnt;          // elements in the interval
  uint64_t w_in;         // weight in the interval
  int32_t action;        // what the next pass does
  int32_t shift;         // digit shift of a refinement pass
  uint32_t res_key;      // result key
  int32_t res_idx;       // result index (or -1)
  uint64_t res_above_w;  // weight strictly above res_key
  uint64_t res_above_c;  // count strictly above res_key
  uint64_t res_cnt_at;   // elements equal to res_key (in the selection's set)
  uint64_t res_w_at;     // weight of one element equal to res_key
  uint64_t aux;          // extra result (rank of the draw inside a tie group, ...)
  int32_t fail;          // no element found for the target (internal error)
};

enum : int32_t { ACT_DONE = 0, ACT_GATHER = 1, ACT_REFINE = 2, ACT_TIE = 3 };
enum : int { MODE_COUNT = 0, MODE_MASS = 1 };

struct alignas(16) Finish {
  int32_t ok, last, n_tie, pad;
  int64_t token;
  uint32_t thr_key, pad2;
  uint64_t zq, kept;
};

struct Shared {
  uint64_t mbar[MAX_STAGE];        // ring stage filled (bulk-copy bytes landed)
  int64_t stage_chunk[MAX_STAGE];  // last chunk issued into each ring stage
  uint32_t released[MAX_STAGE];    // warps done with the chunk in each ring stage
  int32_t cp_flags[3];             // checkpoint flags (timeout 4, overflow 2, crowded 1)
  uint32_t cp_count[3];            // checkpoint: candidates held by the CTA
  // row parameters
  double temperature, top_p;
  uint64_t u53;      // the row's draw as U53 (host uniform or device draw)
  int32_t draw_ok;   // the draw is usable
  int32_t top_k, greedy, filtering, status;
  float tf;
  int64_t row;
  // stage-1 state
  int32_t cand_n, overflow, timeout;
  uint32_t app_n;  // entries of the dense candidate list (rows with a large top_k)
  uint32_t thr;
  float thr_f;
  // published per-CTA stage-1 results (read by the other CTAs of the cluster)
  uint32_t pub_key, pub_idx, pub_min;
  float pub_best, pub_max, pub_mnv;
  float row_best, row_max, row_mnv;
  uint32_t nan_idx;
  int32_t pub_cand_n, pub_overflow, pub_timeout;
  // cluster-wide row facts (identical in every CTA)
  uint32_t mk, arg, kmin;
  int32_t any_overflow, any_timeout;
  // gather list control (rank 0)
  int32_t g_n;
  int32_t nk;
  // decisions
  Dec dec;        // written by rank 0
  Dec dec_local;  // every CTA's copy of rank 0's dec
  Finish fin;
  // scratch for scans and reductions
  uint64_t s64[NW + 2];
  uint32_t s32[NW + 2];
  int32_t found_pos;
  uint64_t found_incl;
  uint32_t red[5 * NW];  // block reductions (sums, maxima, two bisection buffers, minima)
  uint32_t bucket_n, bucket_kth;
  uint32_t bucket[BUCKET];
};

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static constexpr int ES = 4, EPV = 4;
  static constexpr uint32_t NEG_INF_WORD = 0xFF800000u;  // a 32-bit word of -inf elements
  __device__ static float ld(const float* p) { return __ldg(p); }
  // NaN-propagating max of the elements of two words, lane by lane (a word holds 1 or 2 elements)
  __device__ static uint32_t max2(uint32_t a, uint32_t b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(a)), "f"(__uint_as_float(b)));
    return __float_as_uint(r);
  }
  // the largest element of a word, as fp32 (NaN if it holds one)
  __device__ static float word_max(uint32_t w) { return __uint_as_float(w); }
  // element q (runtime index < EPV) of a vector, as fp32
  __device__ static float elem(uint4 v, int q) {
    const uint32_t w = (q & 2) ? ((q & 1) ? v.w : v.z) : ((q & 1) ? v.y : v.x);
    return __uint_as_float(w);
  }
  __device__ static void unpack(uint4 v, float* x) {
    x[0] = __uint_as_float(v.x); x[1] = __uint_as_float(v.y);
    x[2] = __uint_as_float(v.z); x[3] = __uint_as_float(v.w);
  }
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int ES = 2, EPV = 8;
  static constexpr uint32_t NEG_INF_WORD = 0xFF80FF80u;
  __device__ static float ld(const __nv_bfloat16* p) {
    return __uint_as_float(((uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p))) << 16);
  }
  __device__ static uint32_t max2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  __device__ static float word_max(uint32_t w) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(w << 16)), "f"(__uint_as_float(w & 0xFFFF0000u)));
    return r;
  }
  __device__ static float elem(uint4 v, int q) {
    const uint32_t w = (q & 4) ? ((q & 2) ? v.w : v.z) : ((q & 2) ? v.y : v.x);
    return __uint_as_float((q & 1) ? (w & 0xFFFF0000u) : (w << 16));
  }
  __device__ static void unpack(uint4 v, float* x) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};
template <>
struct Elem<__half> {
  static constexpr int ES = 2, EPV = 8;
  static constexpr uint32_t NEG_INF_WORD = 0xFC00FC00u;
  __device__ static float ld(const __half* p) { return __half2float(__ldg(p)); }
  __device__ static uint32_t max2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  __device__ static float word_max(uint32_t w) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;"
        : "=f"(r)
        : "f"(__half2float(__ushort_as_half((unsigned short)(w & 0xFFFF)))),
          "f"(__half2float(__ushort_as_half((unsigned short)(w >> 16)))));
    return r;
  }
  __device__ static float elem(uint4 v, int q) {
    const uint32_t w = (q & 4) ? ((q & 2) ? v.w : v.z) : ((q & 2) ? v.y : v.x);
    return __half2float(__ushort_as_half((unsigned short)((q & 1) ? (w >> 16) : (w & 0xFFFF))));
  }
  __device__ static void unpack(uint4 v, float* x) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xFFFF)));
      x[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    }
  }
};

// This CTA's part of the row: scalar head (rank 0), 16-byte vectors, scalar tail (last rank).
struct Slice {
  int64_t head_n;    // elements [0, head_n) loaded one by one (rank 0 only, else 0)
  int64_t vec_e0;    // first element of this CTA's vectors
  int64_t nvec;      // number of 16-byte vectors
  int64_t tail_e0;   // first tail element (last rank only)
  int64_t tail_n;    // tail elements
  int64_t e_lo, e_hi;  // element range of the whole slice
};

template <typename T>
__device__ Slice make_slice(const T* row, int64_t V, int rank, int C) {
  constexpr int ES = Elem<T>::ES, EPV = Elem<T>::EPV;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(row);
  int64_t head = (int64_t)(((16 - (a0 & 15)) & 15) / ES);
  if (head > V) head = V;
  const int64_t nvec_all = (V - head) / EPV;
  const int64_t tail0 = head + nvec_all * EPV;
  const int64_t base = nvec_all / C, rem = nvec_all % C;
  const int64_t v0 = rank * base + (rank < rem ? rank : rem);
  Slice s;
  s.nvec = base + (rank < rem ? 1 : 0);
  s.vec_e0 = head + v0 * EPV;
  s.head_n = (rank == 0) ? head : 0;
  s.tail_e0 = tail0;
  s.tail_n = (rank == C - 1) ? (V - tail0) : 0;
  s.e_lo = (rank == 0) ? 0 : s.vec_e0;
  s.e_hi = (rank == C - 1) ? V : s.vec_e0 + s.nvec * EPV;
  return s;
}

// Visit every element of the slice (any order per thread; no warp-collective work in f). The
// passes that call this re-read the slice from L2 and do tens of instructions per element, so each
// thread keeps the loads of its next SLICE_AHEAD vectors in flight while it works on one.
constexpr int SLICE_AHEAD = 3;
template <typename T, typename F>
__device__ __forceinline__ void for_slice(const T* row, const Slice& s, F&& f) {
  constexpr int EPV = Elem<T>::EPV;
  for (int64_t e = threadIdx.x; e < s.head_n; e += NT) f(Elem<T>::ld(row + e), (uint32_t)e);
  const uint4* vp = reinterpret_cast<const uint4*>(row + s.vec_e0);
  const uint4 none = make_uint4(0u, 0u, 0u, 0u);
  uint4 ahead[SLICE_AHEAD];
#pragma unroll
  for (int i = 0; i < SLICE_AHEAD; ++i) {
    const int64_t v = threadIdx.x + (int64_t)i * NT;
    ahead[i] = (v < s.nvec) ? __ldg(vp + v) : none;
  }
  for (int64_t v = threadIdx.x; v < s.nvec; v += NT) {
    const uint4 cur = ahead[0];
#pragma unroll
    for (int i = 0; i + 1 < SLICE_AHEAD; ++i) ahead[i] = ahead[i + 1];
    const int64_t vn = v + (int64_t)SLICE_AHEAD * NT;
    ahead[SLICE_AHEAD - 1] = (vn < s.nvec) ? __ldg(vp + vn) : none;
    float x[EPV];
    Elem<T>::unpack(cur, x);
    const uint32_t e0 = (uint32_t)(s.vec_e0 + v * EPV);
#pragma unroll
    for (int j = 0; j < EPV; ++j) f(x[j], e0 + j);
  }
  for (int64_t e = threadIdx.x; e < s.tail_n; e += NT) f(Elem<T>::ld(row + s.tail_e0 + e), (uint32_t)(s.tail_e0 + e));
}

// Visit the slice in index order: tiles of NT consecutive vectors (or scalars for head and tail);
// f(x, e, pred) returns the predicate; g(e, rank_before) is called for every element whose
// predicate holds, with the number of such elements before it in this slice (index order).
template <typename T, typename P, typename G>
__device__ void ordered_slice(const T* row, const Slice& s, Shared& sh, P&& pred, G&& g) {
  constexpr int EPV = Elem<T>::EPV;
  uint32_t run = 0;
  auto scalar_part = [&](int64_t e0, int64_t n) {
    for (int64_t t0 = 0; t0 < n; t0 += NT) {
      const int64_t e = e0 + t0 + threadIdx.x;
      const bool in = (t0 + threadIdx.x) < n;
      float x = in ? Elem<T>::ld(row + e) : 0.0f;
      const uint32_t c = (in && pred(x, (uint32_t)e)) ? 1u : 0u;
      uint32_t tot;
      const uint32_t ex = block_excl_scan<uint32_t, NT>(c, sh.s32, &tot);
      if (c) g(x, (uint32_t)e, run + ex);
      run += tot;
    }
  };
  scalar_part(0, s.head_n);
  const uint4* vp = reinterpret_cast<const uint4*>(row + s.vec_e0);
  for (int64_t t0 = 0; t0 < s.nvec; t0 += NT) {
    const int64_t v = t0 + threadIdx.x;
    float x[EPV];
    bool pr[EPV];
    uint32_t c = 0;
    const uint32_t e0 = (uint32_t)(s.vec_e0 + v * EPV);
    if (v < s.nvec) {
      Elem<T>::unpack(__ldg(vp + v), x);
#pragma unroll
      for (int j = 0; j < EPV; ++j) {
        pr[j] = pred(x[j], e0 + j);
        c += pr[j] ? 1u : 0u;
      }
    } else {
#pragma unroll
      for (int j = 0; j < EPV; ++j) pr[j] = false;
    }
    uint32_t tot;
    uint32_t ex = block_excl_scan<uint32_t, NT>(c, sh.s32, &tot);
    if (c) {
#pragma unroll
      for (int j = 0; j < EPV; ++j)
        if (pr[j]) g(x[j], e0 + j, run + ex++);
    }
    run += tot;
  }
  scalar_part(s.tail_e0, s.tail_n);
}

// Warp-aggregated append of (key, idx) to a shared list; all 32 lanes must call.
__device__ __forceinline__ void warp_append(bool pass, uint32_t key, uint32_t idx, uint64_t* list, int32_t* cnt,
                                            int cap) {
  const uint32_t m = __ballot_sync(0xFFFFFFFFu, pass);
  if (m == 0) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(cnt, __popc(m));
  base = __shfl_sync(0xFFFFFFFFu, base, leader);
  if (pass) {
    const int pos = base + __popc(m & lanemask_lt());
    if (pos < cap) list[pos] = compose(key, idx);
  }
}

// Block-wide (sum, min, max) of one value per thread; every thread gets all three. All threads
// of barrier group B call; the caller separates two calls (and any later use of sh.red) with a barrier.
template <int B = 0>
__device__ __forceinline__ void block_sum_min_max(uint32_t v, uint32_t mn, uint32_t mx, Shared& sh, uint32_t* sum_out,
                                                  uint32_t* min_out, uint32_t* max_out) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = __reduce_add_sync(0xFFFFFFFFu, v);
  mn = __reduce_min_sync(0xFFFFFFFFu, mn);
  mx = __reduce_max_sync(0xFFFFFFFFu, mx);
  if (lane == 0) {
    sh.red[w] = v;
    sh.red[NW + w] = mx;
    sh.red[4 * NW + w] = mn;
  }
  bsync<B>();
  uint32_t s = 0, lo = 0xFFFFFFFFu, hi = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    s += sh.red[i];
    hi = max(hi, sh.red[NW + i]);
    lo = min(lo, sh.red[4 * NW + i]);
  }
  *sum_out = s;
  *min_out = lo;
  *max_out = hi;
}

// k-th largest of the keys the block's threads hold in registers (N per thread), by bisection on
// the key. On entry c_lo = number of held keys >= lo (at least k) and every held key is < hi_excl;
// held keys below lo (fillers) never count. The bisection stops once at most BUCKET keys lie in
// [lo, hi). exact = false returns lo (a lower bound: at least k keys are >= lo, and at most BUCKET
// more than are >= the k-th); exact = true finishes inside the bucket and returns the k-th key
// itself. Every thread returns the same key. All threads of barrier group B call; the caller puts a
// barrier between this and the next use of sh.red.
template <int N, int B = 0>
__device__ uint32_t block_kth_select(const uint32_t (&key)[N], uint32_t k, uint32_t lo, uint32_t c_lo,
                                     uint64_t hi_excl, bool exact, Shared& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint64_t hi = hi_excl;
  uint32_t c_hi = 0;  // held keys >= hi (fewer than k)
  int par = 0;
  while (hi - lo > 1 && c_lo - c_hi > BUCKET) {
    const uint32_t mid = (uint32_t)(lo + ((hi - lo) >> 1));
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < N; ++j) c += (key[j] >= mid) ? 1u : 0u;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if (lane == 0) sh.red[2 * NW + par * NW + w] = c;
    bsync<B>();
    uint32_t tot = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) tot += sh.red[2 * NW + par * NW + i];
    if (tot >= k) {
      lo = mid;
      c_lo = tot;
    } else {
      hi = mid;
      c_hi = tot;
    }
    par ^= 1;
  }
  if (!exact || hi - lo <= 1) return lo;
  // c_lo - c_hi <= BUCKET keys lie in [lo, hi); the answer is the (k - c_hi)-th largest of them
  if (threadIdx.x == 0) sh.bucket_n = 0;
  bsync<B>();
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if (key[j] >= lo && (uint64_t)key[j] < hi) {
      const uint32_t pos = atomicAdd(&sh.bucket_n, 1u);
      if (pos < BUCKET) sh.bucket[pos] = key[j];
    }
  }
  bsync<B>();
  if (w == 0) {
    const uint32_t n = min(sh.bucket_n, BUCKET);
    const uint32_t mine = (uint32_t)lane < n ? sh.bucket[lane] : 0u;
    uint32_t gt = 0, ge = 0;
    for (uint32_t i = 0; i < n; ++i) {
      const uint32_t b = sh.bucket[i];
      gt += (b > mine) ? 1u : 0u;
      ge += (b >= mine) ? 1u : 0u;
    }
    const uint32_t r = k - c_hi;
    const uint32_t hit = __ballot_sync(0xFFFFFFFFu, (uint32_t)lane < n && gt < r && r <= ge);
    if (hit && lane == __ffs(hit) - 1) sh.bucket_kth = mine;  // lanes that hit hold equal keys
  }
  bsync<B>();
  return sh.bucket_kth;
}

// Sort up to 4096 composites descending (bitonic network in shared memory); all threads call.
__device__ void block_sort_desc(uint64_t* a, int n) {
  int N = 2;
  while (N < n) N <<= 1;
  for (int i = n + threadIdx.x; i < N; i += NT) a[i] = 0;  // pads sort last
  __syncthreads();
  for (int k = 2; k <= N; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < (N >> 1); i += NT) {
        const int lo = 2 * i - (i & (j - 1));
        const int hi = lo + j;
        const uint64_t x = a[lo], y = a[hi];
        const bool desc = (lo & k) == 0;
        if (desc ? (x < y) : (x > y)) {
          a[lo] = y;
          a[hi] = x;
        }
      }
      __syncthreads();
    }
  }
}

// Over a sorted list a[0..n): weights q (mode MASS) or 1 (mode COUNT); find the first position whose
// inclusive prefix (plus `base`) exceeds `target`. Writes sh.found_pos / sh.found_incl
// (found_incl = base + inclusive prefix at the position). All threads call.
__device__ void list_find(const uint64_t* a, int n, int mode, float m, uint64_t base, uint64_t target, Shared& sh) {
  const int seg = (n + NT - 1) / NT;
  const int p0 = min(n, (int)threadIdx.x * seg), p1 = min(n, p0 + seg);
  uint64_t sum = 0;
  for (int p = p0; p < p1; ++p) sum += (mode == MODE_MASS) ? weight_q(value_of(comp_key(a[p])), m) : 1ull;
  uint64_t tot;
  const uint64_t ex = block_excl_scan<uint64_t, NT>(sum, sh.s64, &tot);
  if (threadIdx.x == 0) sh.found_pos = -1;
  __syncthreads();
  const uint64_t lo = base + ex;
  if (lo <= target && target < lo + sum) {
    uint64_t run = lo;
    for (int p = p0; p < p1; ++p) {
      run += (mode == MODE_MASS) ? weight_q(value_of(comp_key(a[p])), m) : 1ull;
      if (run > target) {
        sh.found_pos = p;
        sh.found_incl = run;
        break;
      }
    }
  }
  __syncthreads();
}

// first position p in sorted a[0..n) with comp_key(a[p]) == key (keys descending); single thread
__device__ int first_of_key(const uint64_t* a, int n, uint32_t key) {
  int lo = 0, hi = n;  // first p with comp_key(a[p]) <= key
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (comp_key(a[mid]) > key) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}


// Resolve a small survivor set in one warp: sort (key desc, index asc), fixed-point weights,
// inclusive scan, top-p cut and the draw. n <= 64; lanes 0..31 of one warp call.
__device__ void warp_finish(uint64_t* K, int n, float m, bool topp, float pf, uint64_t u53, Finish* f) {
  const int lane = threadIdx.x & 31;
  // bitonic sort of the (up to) 64 composites, descending, in registers: lane l holds positions
  // 2l (a) and 2l + 1 (b); padding (0) sorts last
  uint64_t a = (2 * lane < n) ? K[2 * lane] : 0ull;
  uint64_t b = (2 * lane + 1 < n) ? K[2 * lane + 1] : 0ull;
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const bool desc = ((2 * lane) & k) == 0;  // the same for both positions of a lane (k >= 2)
      if (j == 1) {
        if (desc ? (a < b) : (a > b)) {
          const uint64_t t = a;
          a = b;
          b = t;
        }
      } else {
        const bool lower = ((2 * lane) & j) == 0;  // partner positions differ by j: lanes by j / 2
        const uint64_t oa = __shfl_xor_sync(0xFFFFFFFFu, a, j >> 1);
        const uint64_t ob = __shfl_xor_sync(0xFFFFFFFFu, b, j >> 1);
        a = (lower == desc) ? max(a, oa) : min(a, oa);
        b = (lower == desc) ? max(b, ob) : min(b, ob);
      }
    }
  }
  K[2 * lane] = a;
  K[2 * lane + 1] = b;
  __syncwarp();
  const uint64_t qa = (2 * lane < n) ? weight_q(value_of(comp_key(a)), m) : 0ull;
  const uint64_t qb = (2 * lane + 1 < n) ? weight_q(value_of(comp_key(b)), m) : 0ull;
  const uint64_t s = qa + qb;
  const uint64_t incl = warp_incl_scan(s);
  const uint64_t excl = incl - s;
  const uint64_t zq = __shfl_sync(0xFFFFFFFFu, incl, 31);
  // first position whose inclusive prefix exceeds t (t < total)
  auto find = [&](uint64_t t, uint64_t* at) -> int {
    const bool here = excl <= t && t < incl;
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, here);
    if (bal == 0) return -1;
    const int src = __ffs(bal) - 1;
    const int pos = (excl + qa > t) ? 2 * lane : 2 * lane + 1;
    const uint64_t inc = (excl + qa > t) ? excl + qa : incl;
    *at = __shfl_sync(0xFFFFFFFFu, inc, src);
    return __shfl_sync(0xFFFFFFFFu, pos, src);
  };
  int last = n - 1;
  uint64_t kept = zq;
  bool ok = n > 0;
  if (ok && topp) {
    last = find(mul_floor(pf, zq), &kept);
    ok = last >= 0;
  }
  int pick = -1;
  if (ok) {
    uint64_t dummy;
    pick = find(scale_u53(u53, kept), &dummy);
    ok = pick >= 0;
  }
  if (!ok) {
    last = 0;
    pick = 0;
  }
  const uint32_t tk = comp_key(K[last]);
  const int c = ((2 * lane <= last && comp_key(a) == tk) ? 1 : 0) + ((2 * lane + 1 <= last && comp_key(b) == tk) ? 1 : 0);
  const int n_tie = warp_sum(c);
  if (lane == 0) {
    f->ok = ok;
    f->last = last;
    f->n_tie = n_tie;
    f->token = ok ? (int64_t)comp_idx(K[pick]) : -1;
    f->thr_key = tk;
    f->zq = zq;
    f->kept = kept;
  }
}

__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Smallest raw value r with key(r / T) >= key(t / T): raw values at or above it are exactly the
// ones whose scaled key reaches t's scaled key (division can merge neighbouring raw values).
// Steps down from t one raw value at a time (at most 64 steps, divisions of ordinary values only);
// when t is not an ordinary value or the step limit is reached it returns -inf, which keeps every
// value (still exact, only less selective).
__device__ float tie_floor(float t, float tf) {
  const float at = fabsf(t);
  if (!(at >= 0x1p-100f && at <= 0x1p100f) || !(tf >= 0x1p-60f && tf <= 0x1p60f)) return -INFINITY;
  const uint32_t target = key_of(__fdiv_rn(t, tf));
  uint32_t u = key_of(t);
  for (int i = 0; i < 64; ++i) {
    const float below = value_of(u - 1);
    if (!(fabsf(below) >= 0x1p-100f)) return -INFINITY;
    if (key_of(__fdiv_rn(below, tf)) < target) return value_of(u);
    --u;
  }
  return -INFINITY;
}

// 1 / t when t is a power of two whose reciprocal is a normal float (then exact), else 0
__device__ __forceinline__ float exact_reciprocal(float t) {
  const uint32_t b = __float_as_uint(t);
  const uint32_t e = (b >> 23) & 0xFF;
  if ((b & 0x807FFFFFu) != 0 || e < 1 || e > 253) return 0.0f;
  return __uint_as_float((254u - e) << 23);
}

// level-1 bin of a key: distance below the max, scaled; non-increasing in the key
__device__ __forceinline__ int bin_of(float key, float m, float scale) {
  const float v = __fmul_rn(-__fsub_rn(key, m), scale);
  return (v < (float)NBIN) ? (int)v : NBIN - 1;
}
__device__ __forceinline__ int bin_of_key(uint32_t k, float m, float scale) { return bin_of(value_of(k), m, scale); }

// key interval [lo, hi] (within [0, mk]) of level-1 bin b
__device__ void bin_interval(int b, uint32_t mk, float m, float scale, uint32_t* lo, uint32_t* hi) {
  auto first_le = [&](int bb) -> uint32_t {  // smallest key in [0, mk] whose bin <= bb
    uint32_t a = 0, z = mk;
    while (a < z) {
      const uint32_t mid = a + ((z - a) >> 1);
      if (bin_of_key(mid, m, scale) <= bb) z = mid;
      else a = mid + 1;
    }
    return a;
  };
  *lo = first_le(b);
  *hi = (b == 0) ? mk : first_le(b - 1) - 1;
}

// ---- cluster helpers ------------------------------------------------------------------------

__device__ __forceinline__ void pull_dec(cg::cluster_group& cluster, Shared& sh) {
  if (threadIdx.x == 0) {
    const Dec* d = cluster.map_shared_rank(&sh.dec, 0);
    sh.dec_local = *d;
  }
  __syncthreads();
}

// Rank 0 sums the C CTAs' histograms into its own (hq/hc) and finds the bin whose inclusive
// prefix of weight exceeds `target`. Weight = hq (MASS) or hc (COUNT). All rank-0 threads call.
__device__ void reduce_and_find(cg::cluster_group& cluster, int C, uint64_t* hq, uint32_t* hc, uint64_t* out_q,
                                uint32_t* out_c, int nbins, int mode, uint64_t target, Shared& sh, int* b_out,
                                uint64_t* above_w, uint64_t* above_c, uint64_t* bin_w, uint64_t* bin_c) {
  for (int b = threadIdx.x; b < nbins; b += NT) {
    uint64_t q = 0;
    uint32_t c = 0;
    for (int r = 0; r < C; ++r) {
      const uint64_t* rq = cluster.map_shared_rank(hq, r);
      const uint32_t* rc = cluster.map_shared_rank(hc, r);
      if (mode == MODE_MASS) q += rq[b];
      c += rc[b];
    }
    out_q[b] = (mode == MODE_MASS) ? q : (uint64_t)c;
    out_c[b] = c;
  }
  __syncthreads();
  const int per = (nbins + NT - 1) / NT;
  const int b0 = min(nbins, (int)threadIdx.x * per), b1 = min(nbins, b0 + per);
  uint64_t sw = 0, sc = 0;
  for (int b = b0; b < b1; ++b) {
    sw += out_q[b];
    sc += out_c[b];
  }
  uint64_t tw, tc;
  const uint64_t ew = block_excl_scan<uint64_t, NT>(sw, sh.s64, &tw);
  const uint64_t ec = block_excl_scan<uint64_t, NT>(sc, sh.s64, &tc);
  if (threadIdx.x == 0) sh.found_pos = -1;
  __syncthreads();
  if (ew <= target && target < ew + sw) {
    uint64_t rw = ew, rc = ec;
    for (int b = b0; b < b1; ++b) {
      if (rw + out_q[b] > target) {
        sh.found_pos = b;
        sh.s64[NW + 1] = rw;  // above weight
        sh.found_incl = rc;   // above count
        break;
      }
      rw += out_q[b];
      rc += out_c[b];
    }
  }
  __syncthreads();
  *b_out = sh.found_pos;
  if (sh.found_pos >= 0) {
    *above_w = sh.s64[NW + 1];
    *above_c = sh.found_incl;
    *bin_w = out_q[sh.found_pos];
    *bin_c = out_c[sh.found_pos];
  }
  __syncthreads();
}

// Lower bound of the k-th largest key the CTA holds when every thread offers one key it holds (0:
// none): each warp sorts its 32 offers (bitonic, in registers), takes its ceil(k / NW)-th largest,
// and the CTA takes the smallest of those, so the NW warps hold at least k keys at or above it.
// k <= OFFER_KMAX. Every thread returns the same key. All threads of barrier group B call; the
// caller separates two calls (and any other use of sh.red[3 * NW ...]) with a barrier.
constexpr int OFFER_KMAX = 32 * NW;
// k up to which thresholds come from the offer bound (above it the bound, the smallest of a few
// offers per warp, is too loose to thin candidates out; an exact bisection takes those)
constexpr int OFFER_PREFER = 16 * NW;
template <int B = 0>
__device__ uint32_t block_offer_bound(uint32_t key, int k, Shared& sh) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, key, stride);
      const bool desc = (lane & size) == 0;
      const bool lower = (lane & stride) == 0;
      key = (lower == desc) ? max(key, o) : min(key, o);
    }
  }
  const uint32_t kj = __shfl_sync(0xFFFFFFFFu, key, (k + NW - 1) / NW - 1);
  if (lane == 0) sh.red[3 * NW + w] = kj;
  bsync<B>();
  uint32_t mn = 0xFFFFFFFFu;
#pragma unroll
  for (int i = 0; i < NW; ++i) mn = min(mn, sh.red[3 * NW + i]);
  return mn;
}

// Warp-aggregated append of a candidate (raw value x, index e) to the CTA's dense candidate list
// (entry i sits in slot i / NT of thread i % NT, the layout compact_slots repacks to). All 32 lanes
// call. Returns false for a lane whose candidate found no room.
__device__ __forceinline__ bool append_dense(bool pass, float x, uint32_t e, uint64_t* list, uint32_t* cnt) {
  const uint32_t m = __ballot_sync(0xFFFFFFFFu, pass);
  if (m == 0) return true;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  uint32_t base = 0;
  if (lane == leader) base = atomicAdd(cnt, (uint32_t)__popc(m));
  base = __shfl_sync(0xFFFFFFFFu, base, leader);
  if (!pass) return true;
  const uint32_t pos = base + (uint32_t)__popc(m & lanemask_lt());
  if (pos >= (uint32_t)CAND_CAP) return false;
  list[pos] = compose(key_of(x), e);
  return true;
}

// slots a thread holds of a dense list of n entries
__device__ __forceinline__ int dense_slots(uint32_t n) {
  const uint32_t t = threadIdx.x;
  return (n > t) ? (int)min((uint32_t)SLOTS, (n - t + NT - 1) / NT) : 0;
}

// ---- the kernel -------------------------------------------------------------------------

// Raise the candidate threshold sh.thr_f to the tie floor of a lower bound of the kth_rank-th
// largest candidate held in the per-thread slots (slot j of thread t at candB[j * NT + t]) and
// drop the candidates below it. Returns this thread's new slot count. All threads of barrier group
// B call; a barrier separates two calls. Kept out of line so the streaming loop stays small.
template <int B = 0>
__device__ __noinline__ int compact_slots(uint64_t* candB, int nc, int kth_rank, float tf, Shared& sh,
                                         uint32_t* count_out = nullptr) {
  const int tid = threadIdx.x;
  if (kth_rank <= OFFER_PREFER) {
    // every thread offers its largest candidate; the bound only ever raises the threshold
    uint32_t top = 0;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j)
      if (j < nc) top = max(top, comp_key(candB[j * NT + tid]));
    const uint32_t lo = block_offer_bound<B>(top, kth_rank, sh);
    const float old = sh.thr_f;
    bsync<B>();  // every thread has read the old threshold and sh.red
    if (tid == 0 && lo > KEY_NEG_INF) sh.thr_f = fmaxf(old, tie_floor(value_of(lo), tf));
    bsync<B>();
    const uint32_t fk = key_of(sh.thr_f);
    int w = 0;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j) {
      if (j < nc) {
        const uint64_t c = candB[j * NT + tid];
        if (comp_key(c) >= fk) {
          candB[w * NT + tid] = c;
          ++w;
        }
      }
    }
    return w;
  }
  uint32_t kk[SLOTS];
  uint32_t mn = 0xFFFFFFFFu, mx = 0;
#pragma unroll
  for (int j = 0; j < SLOTS; ++j) {
    kk[j] = (j < nc) ? comp_key(candB[j * NT + tid]) : 0u;
    if (j < nc) mn = min(mn, kk[j]);
    mx = max(mx, kk[j]);
  }
  uint32_t tot, kmin, kmax;
  block_sum_min_max<B>((uint32_t)nc, mn, mx, sh, &tot, &kmin, &kmax);
  if ((int)tot < kth_rank) return nc;  // fewer candidates than k: nothing to raise
  // a lower bound of the kth_rank-th candidate (at most BUCKET more candidates above it)
  const uint32_t kth_raw =
      block_kth_select<SLOTS, B>(kk, (uint32_t)kth_rank, kmin, tot, (uint64_t)kmax + 1, false, sh);
  bsync<B>();  // every thread has read the old threshold
  if (tid == 0) sh.thr_f = tie_floor(value_of(kth_raw), tf);
  bsync<B>();
  const uint32_t fk = key_of(sh.thr_f);
  // A large k keeps about k candidates, and a thread may hold many of them: deal the kept ones out
  // evenly (entry i of the dense list goes to slot i / NT of thread i % NT), so that no thread
  // stays crowded with candidates the new threshold cannot drop.
  uint64_t v[SLOTS];
  uint32_t keep = 0;
#pragma unroll
  for (int j = 0; j < SLOTS; ++j) {
    v[j] = (j < nc) ? candB[j * NT + tid] : 0ull;
    keep += (j < nc && kk[j] >= fk) ? 1u : 0u;
  }
  uint32_t kept;
  uint32_t pos = block_excl_scan<uint32_t, NT, B>(keep, sh.s32, &kept);  // every slot is read first
#pragma unroll
  for (int j = 0; j < SLOTS; ++j) {
    if (j < nc && kk[j] >= fk) candB[pos++] = v[j];
  }
  if (count_out && tid == 0) *count_out = kept;
  bsync<B>();
  return (kept > (uint32_t)tid) ? (int)((kept - (uint32_t)tid + NT - 1) / NT) : 0;
}

// First candidate threshold: sh.thr_f = the tie floor of the top_k-th largest value among the nv
// staged vectors at buf (thread t owns vectors t, t + NT, ...). All threads call.
// First candidate threshold, a lower bound of the row's top_k-th value taken from the nv staged
// vectors at buf (thread t owns vectors t, t + NT, ...): the top_k-th largest per-thread maximum
// when at least top_k threads hold values (every maximum is a value of the row), else the
// top_k-th largest value. sh.thr_f = its tie floor. All threads call.
template <typename T, int VPT>
__device__ __noinline__ void first_threshold(const uint4* buf, int nv, int top_k, float tf, Shared& sh) {
  constexpr int EPV = Elem<T>::EPV;
  const int tid = threadIdx.x;
  uint32_t kk[VPT * EPV];
  uint32_t mn = 0xFFFFFFFFu, mx = 0, tmax = 0;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const bool ok = j * NT + tid < nv;
    float x[EPV];
    if (ok) Elem<T>::unpack(buf[j * NT + tid], x);
#pragma unroll
    for (int q = 0; q < EPV; ++q) {
      kk[j * EPV + q] = ok ? key_of(x[q]) : 0u;
      if (ok) mn = min(mn, kk[j * EPV + q]);
      mx = max(mx, kk[j * EPV + q]);
    }
  }
  tmax = mx;  // this thread's maximum key (0 if it holds no value)
  const int holders = min(nv, NT);
  uint32_t k0;
  if (top_k <= OFFER_PREFER) {
    k0 = block_offer_bound(tmax, top_k, sh);
    __syncthreads();  // sh.red read by every thread
    if (tid == 0) sh.thr_f = (k0 > KEY_NEG_INF) ? tie_floor(value_of(k0), tf) : -INFINITY;
    __syncthreads();
    return;
  }
  if (holders >= top_k) {
    uint32_t one[1] = {tmax};
    uint32_t unused, tmin, tmx;
    block_sum_min_max(0u, tmax ? tmax : 0xFFFFFFFFu, tmax, sh, &unused, &tmin, &tmx);
    k0 = block_kth_select<1>(one, (uint32_t)top_k, tmin, (uint32_t)holders, (uint64_t)tmx + 1, false, sh);
  } else {
    uint32_t unused, kmin, kmax;
    block_sum_min_max(0u, mn, mx, sh, &unused, &kmin, &kmax);
    k0 = block_kth_select<VPT * EPV>(kk, (uint32_t)top_k, kmin, (uint32_t)(nv * EPV), (uint64_t)kmax + 1, false, sh);
  }
  if (tid == 0) sh.thr_f = tie_floor(value_of(k0), tf);
  __syncthreads();
}

// Resolve the survivor list K[0..nk) (composites of scaled key and index, any order, nk <= KCAP)
// in one CTA: order (key desc, index asc), fixed-point weights, top-p cut, draw. Thread 0 gets the
// token and the kept-set description; every thread gets sh.found_pos (last kept position) and
// sh.s64[NW + 1] (kept mass) for the probability write. All threads call.
__device__ void finish_survivors(uint64_t* K, int nk, float m, bool topp_active, float pf, uint64_t u53, Shared& sh,
                                 int64_t* token, pb_row_info* info) {
  const int tid = threadIdx.x;
  if (nk <= 64) {
    Finish f;
    if (tid < 32) warp_finish(K, nk, m, topp_active, pf, u53, &f);
    if (tid == 0) sh.fin = f;
    __syncthreads();
    f = sh.fin;
    if (tid == 0) {
      if (!f.ok) info->status = PB_ROW_INTERNAL;
      *token = f.token;
      info->thr_key = f.thr_key;
      info->n_tie_kept = f.n_tie;
      info->kept_count = f.last + 1;
      info->z_q = f.zq;
      info->kept_q = f.kept;
      info->flags = PB_PATH_SMALL;
      sh.nk = nk;
      sh.found_pos = f.last;
      sh.s64[NW + 1] = f.kept;
    }
    __syncthreads();
    return;
  }
  block_sort_desc(K, nk);
  uint64_t zq;
  {
    const int seg = (nk + NT - 1) / NT;
    const int p0 = min(nk, tid * seg), p1 = min(nk, p0 + seg);
    uint64_t sum = 0;
    for (int p = p0; p < p1; ++p) sum += weight_q(value_of(comp_key(K[p])), m);
    block_excl_scan<uint64_t, NT>(sum, sh.s64, &zq);
  }
  int last = nk - 1;
  uint64_t kept = zq;
  bool ok = true;
  if (topp_active) {
    list_find(K, nk, MODE_MASS, m, 0, mul_floor(pf, zq), sh);
    last = sh.found_pos;
    kept = sh.found_incl;
    ok = last >= 0;
  }
  int pick = -1;
  if (ok) {
    list_find(K, nk, MODE_MASS, m, 0, scale_u53(u53, kept), sh);
    pick = sh.found_pos;
    ok = pick >= 0;
  }
  if (!ok) {
    last = 0;
    pick = 0;
    if (tid == 0) info->status = PB_ROW_INTERNAL;
  }
  __syncthreads();  // every thread has read sh.found_pos
  if (tid == 0) {
    *token = comp_idx(K[pick]);
    const uint32_t tk = comp_key(K[last]);
    info->thr_key = tk;
    info->n_tie_kept = last - first_of_key(K, nk, tk) + 1;
    info->kept_count = last + 1;
    info->z_q = zq;
    info->kept_q = kept;
    info->flags = PB_PATH_SMALL;
    sh.nk = nk;
    sh.found_pos = last;
    sh.s64[NW + 1] = kept;
  }
  __syncthreads();
}

#include "pb_stream.cuh"
#include "pb_groups.cuh"

template <typename T>
__global__ void __launch_bounds__(NT, 2) sample_kernel(Args a) {
  constexpr int ES = Elem<T>::ES, EPV = Elem<T>::EPV;
  constexpr int CHUNK_VEC = CHUNK_BYTES / 16;
  constexpr int VPT = CHUNK_VEC / NT;  // vectors per thread per chunk
  constexpr int NSTAGE = RING_BYTES / CHUNK_BYTES;
  (void)ES;
  static_assert(CHUNK_VEC % NT == 0, "chunk must split evenly");

  extern __shared__ __align__(128) unsigned char dyn[];
  __shared__ Shared sh;
  unsigned char* regA = dyn;
  uint64_t* candB = reinterpret_cast<uint64_t*>(dyn + REGION_A);
  uint64_t* h1q = reinterpret_cast<uint64_t*>(regA + NBIN * 12);
  uint32_t* h1c = reinterpret_cast<uint32_t*>(regA + NBIN * 20);
  uint64_t* hq = reinterpret_cast<uint64_t*>(regA);
  uint32_t* hc = reinterpret_cast<uint32_t*>(regA + NBIN * 8);

  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  // cluster barrier; a one-CTA cluster needs only the CTA barrier (same ordering, far cheaper)
  auto csync = [&]() {
    if (C == 1) __syncthreads();
    else cluster.sync();
  };
  const int64_t item = blockIdx.x / C;
  const int tid = threadIdx.x;
  const int64_t V = a.vocab;
  // rows another launch already settled: every CTA of the cluster leaves before any cluster step
  if (a.only_fallback && a.only_fallback[item].status != PB_ROW_FALLBACK) return;
  if (a.complement && fast_mode(a.params[item], V) != F_NONE) {
    // the streaming kernel took this row; it left a mark if it could not settle it
    griddep_wait();
    const bool retry = a.cand_out ? reinterpret_cast<const pb_cand_header*>(a.cand_out + item * record_bytes(a.cand_cap))
                                            ->flags == F_CAND_RETRY
                                  : a.out_token[item] == F_RETRY;
    if (!retry) return;
  }

  if (tid == 0) {
    const pb_row_params p = a.params[item];
    sh.temperature = p.temperature;
    sh.top_p = p.top_p;
    sh.u53 = row_u53(p);
    sh.draw_ok = row_draw_ok(p) ? 1 : 0;
    sh.top_k = p.top_k;
    sh.greedy = (p.temperature == 0.0);
    sh.tf = (float)p.temperature;
    sh.filtering = !sh.greedy && p.top_k > 0 && (int64_t)p.top_k < V && p.top_k <= KSMALL;
    sh.row = a.row_index ? (int64_t)a.row_index[item] : item;
    sh.cand_n = 0;
    sh.app_n = 0;
    sh.overflow = 0;
    sh.timeout = 0;
    sh.thr = 0;
    sh.thr_f = -INFINITY;
    sh.status = PB_ROW_OK;
    // parameters the reference's SamplingParams rejects (config.py:146-155)
    const bool bad = !(p.temperature >= 0.0) || !(p.top_p > 0.0 && p.top_p <= 1.0) || p.top_k < 0;
    if (bad) {
      sh.status = PB_ROW_BAD_PARAMS;
      sh.filtering = 0;
    }
    for (int st = 0; st < NSTAGE; ++st) {
      mbar_init(&sh.mbar[st], 1);
      sh.stage_chunk[st] = -1;
      sh.released[st] = 0;
    }
    sh.cp_flags[0] = sh.cp_flags[1] = sh.cp_flags[2] = 0;
    sh.cp_count[0] = sh.cp_count[1] = sh.cp_count[2] = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const bool greedy = sh.greedy;
  const bool filtering = sh.filtering;
  const float tf = sh.tf;
  // x / T per element (the cooperative path's passes): a power-of-two T has an exact reciprocal,
  // and then x * (1 / T) rounds the same real number as x / T, so it is the same float for a
  // fraction of the cost
  const float t_inv = exact_reciprocal(tf);
  auto scaled = [&](float x) { return (t_inv != 0.0f) ? __fmul_rn(x, t_inv) : __fdiv_rn(x, tf); };
  const int32_t top_k = sh.top_k;
  const T* row = reinterpret_cast<const T*>(a.logits) + sh.row * a.row_stride;
  const Slice s = make_slice(row, V, rank, C);

  // ---------------- stage 1: stream the slice ----------------
  // Raw values are compared directly (x / T is monotone in x for T > 0): a NaN-propagating max,
  // the first (lowest-index) maximum, the smallest value above -inf for rows that need it, and for
  // small top-k rows the candidates (raw value >= a running threshold) in per-thread slots.
  // Each thread handles VPT independent 16-byte vectors per 32 KB chunk.
  const bool track_min = !greedy && !filtering;  // rows that take the cooperative path
  float runmax = -INFINITY, bestv = -INFINITY, mnv = INFINITY;
  uint32_t bidx = 0xFFFFFFFFu;
  int nc = 0;             // this thread's occupied candidate slots
  bool ovf = false;       // a candidate of this thread found no free slot
  bool row_ovf = false;   // some thread of the CTA overflowed (uniform: from __syncthreads_or)

  auto push = [&](float x, uint32_t e) {
    if (nc < SLOTS) {
      candB[nc * NT + tid] = compose(key_of(x), e);
      ++nc;
    } else {
      ovf = true;
    }
  };
  // Raise the threshold to the tie floor of the kth_rank-th largest candidate and drop the
  // candidates below it (each thread compacts its own slots). All threads call; a barrier
  // separates two calls.
  // Rows with a large top_k pass about k values per chunk and keep about k: their candidates go to
  // one dense list of the CTA (warp-aggregated appends), so no thread's slots overflow first.
  const bool dense_mode = filtering && top_k > OFFER_PREFER;
  auto compact = [&](int kth_rank) {
    nc = compact_slots(candB, nc, kth_rank, tf, sh, dense_mode ? &sh.app_n : nullptr);
  };
  auto visit1 = [&](float x, uint32_t e) {
    runmax = fmax_nan(runmax, x);
    if (x > bestv) {
      bestv = x;
      bidx = e;
    }
    if (track_min && x > -INFINITY) mnv = fminf(mnv, x);
  };

  // scalar head (rank 0): max only; filtered after the stream against the final threshold
  for (int64_t e = tid; e < s.head_n; e += NT) visit1(Elem<T>::ld(row + e), (uint32_t)e);
  {
    const int64_t nchunks = (s.nvec + CHUNK_VEC - 1) / CHUNK_VEC;
    const uint4* src = reinterpret_cast<const uint4*>(row + s.vec_e0);
    uint4* ring = reinterpret_cast<uint4*>(regA);
    const bool keep_in_l2 = !greedy && !filtering;  // rows that re-read their slice
    // Warps consume the ring independently: each waits on a stage's full barrier, copies its
    // vectors to registers and releases the stage; the last warp to release it issues the next
    // copy into it. The CTA meets only at checkpoints (every NSTAGE chunks and after the last),
    // where it agrees on timeouts, candidate overflow and crowded slots (then compacts).
    auto issue = [&](int64_t c) {
      const int st = (int)(c % NSTAGE);
      const uint64_t pol = keep_in_l2 ? l2_policy_evict_last() : l2_policy_evict_first();
      const int64_t nv = min((int64_t)CHUNK_VEC, s.nvec - c * CHUNK_VEC);
      sh.stage_chunk[st] = c;
      mbar_expect_tx(&sh.mbar[st], (uint32_t)(nv * 16));
      bulk_load(ring + st * CHUNK_VEC, src + c * CHUNK_VEC, (uint32_t)(nv * 16), &sh.mbar[st], pol);
    };
    if (tid == 0)
      for (int64_t c = 0; c < NSTAGE && c < nchunks; ++c) issue(c);
    const int lane = tid & 31;
    bool timed_out = false;  // this warp gave up waiting (warp-uniform)
    if (filtering && nchunks > 0) {
      // first threshold from the first chunk (it stays staged for the loop below)
      timed_out = !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&sh.mbar[0], 0u, WAIT_POLLS));
      const int nv0 = (int)min((int64_t)CHUNK_VEC, s.nvec);
      if (nv0 * EPV >= top_k) first_threshold<T, VPT>(ring, nv0, top_k, tf, sh);
    }
    bool cta_timeout = false;
    int cp = 0;              // checkpoints passed
    // A large k passes about k values per chunk past a threshold taken from the first chunk, so the
    // slots fill within a few chunks: such rows meet (and may compact) after every chunk.
    const int cp_every = (filtering && top_k > OFFER_PREFER) ? 1 : CP_CHUNKS;
    // 32-bit chunk and vector counters: a slice holds fewer than 2^24 elements
    const int nch = (int)nchunks, nvec32 = (int)s.nvec;
    const uint32_t e_base = (uint32_t)s.vec_e0 + (uint32_t)tid * EPV;  // element of vector tid of chunk 0
    float t = sh.thr_f;  // candidate threshold; changes only at checkpoints
    for (int c = 0; c < nch; ++c) {
      const int stage = c % NSTAGE;
      const uint32_t parity = (uint32_t)((c / NSTAGE) & 1);
      if (!timed_out) timed_out = !__all_sync(0xFFFFFFFFu, mbar_wait_bounded(&sh.mbar[stage], parity, WAIT_POLLS));
      const int nv = min(CHUNK_VEC, nvec32 - c * CHUNK_VEC);
      const uint4* buf = ring + stage * CHUNK_VEC;
      // load every vector of this thread first (independent shared loads), then reduce
      float x[VPT][EPV];
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = j * NT + tid;
        if (v < nv && !timed_out) {
          Elem<T>::unpack(buf[v], x[j]);
        } else {
#pragma unroll
          for (int q = 0; q < EPV; ++q) x[j][q] = -INFINITY;
        }
      }
      __syncwarp();
      if (lane == 0 && !timed_out) {
        // this warp is done with the stage; the last warp to release it refills it
        if (atom_add_acq_rel(&sh.released[stage], 1u) == NW - 1) {
          sh.released[stage] = 0;
          if (c + NSTAGE < nch) {
            fence_proxy_async();
            issue(c + NSTAGE);
          }
        }
      }
      float vm[VPT];
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        float a = fmax_nan(x[j][0], x[j][1]);
#pragma unroll
        for (int q = 2; q < EPV; ++q) a = fmax_nan(a, x[j][q]);
        vm[j] = a;
      }
#pragma unroll
      for (int j = 0; j < VPT; ++j) runmax = fmax_nan(runmax, vm[j]);
      if (greedy) {  // only greedy rows need the index of the first maximum
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          if (vm[j] > bestv) {
            bestv = vm[j];
            int jj = EPV - 1;
#pragma unroll
            for (int q = EPV - 1; q >= 0; --q)
              if (x[j][q] == vm[j]) jj = q;
            bidx = e_base + (uint32_t)((c * CHUNK_VEC + j * NT) * EPV + jj);
          }
        }
      }
      if (track_min) {
#pragma unroll
        for (int j = 0; j < VPT; ++j)
#pragma unroll
          for (int q = 0; q < EPV; ++q)
            if (x[j][q] > -INFINITY) mnv = fminf(mnv, x[j][q]);
      }
      if (filtering && !row_ovf && dense_mode) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const bool any = j * NT + tid < nv && vm[j] >= t;
          if (__any_sync(0xFFFFFFFFu, any)) {
            const uint32_t e0 = e_base + (uint32_t)((c * CHUNK_VEC + j * NT) * EPV);
#pragma unroll
            for (int q = 0; q < EPV; ++q)
              if (!append_dense(any && x[j][q] >= t, x[j][q], e0 + q, candB, &sh.app_n)) ovf = true;
          }
        }
      } else if (filtering && !row_ovf) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          if (j * NT + tid < nv && vm[j] >= t) {  // vectors past the chunk's end hold -inf padding
            const uint32_t e0 = e_base + (uint32_t)((c * CHUNK_VEC + j * NT) * EPV);
#pragma unroll
            for (int q = 0; q < EPV; ++q)
              if (x[j][q] >= t) push(x[j][q], e0 + q);
          }
        }
      }
      if ((c + 1) % cp_every == 0 || c == nch - 1) {
        // checkpoint; flag and count words rotate over three slots so a reset never races a write
        const int mine =
            (timed_out ? 4 : 0) | (ovf ? 2 : 0) | ((filtering && !dense_mode && nc >= SLOTS / 2) ? 1 : 0);
        if (mine) atomicOr(&sh.cp_flags[cp % 3], mine);
        if (filtering && !dense_mode) {
          const uint32_t wsum = __reduce_add_sync(0xFFFFFFFFu, (uint32_t)nc);
          if (lane == 0 && wsum) atomicAdd(&sh.cp_count[cp % 3], wsum);
        }
        __syncthreads();
        const int f = sh.cp_flags[cp % 3];
        const uint32_t held = dense_mode ? sh.app_n : sh.cp_count[cp % 3];
        // every thread reads the dense count before any warp appends again (one decision per CTA)
        if (dense_mode) __syncthreads();
        if (tid == 0) {
          sh.cp_flags[(cp + 2) % 3] = 0;
          sh.cp_count[(cp + 2) % 3] = 0;
        }
        ++cp;
        if (f & 4) {
          cta_timeout = true;
          break;
        }
        if (f & 2) row_ovf = true;
        // raise the threshold once the CTA holds a few times k candidates, so it keeps tracking
        // the k-th of everything seen (the pass rate then falls with the chunks streamed)
        if (((f & 1) || held >= (uint32_t)((dense_mode ? 2 : 4) * top_k + 64)) && !row_ovf) {
          if (dense_mode) nc = dense_slots(held);  // no overflow: held <= CAND_CAP
          compact(top_k);
        }
        t = sh.thr_f;  // every thread passed the barrier after any write of the threshold
      }
    }
    if (cta_timeout) {
      // let every issued copy land before the shared memory is reused
      if (tid == 0) {
        sh.timeout = 1;
        for (int st = 0; st < NSTAGE; ++st) {
          const int64_t c = sh.stage_chunk[st];
          if (c >= 0) mbar_wait_bounded(&sh.mbar[st], (uint32_t)((c / NSTAGE) & 1), WAIT_POLLS);
        }
      }
      __syncthreads();
    }
  }
  for (int64_t e = tid; e < s.tail_n; e += NT) visit1(Elem<T>::ld(row + s.tail_e0 + e), (uint32_t)(s.tail_e0 + e));
  if (filtering) {
    // head and tail elements against the final threshold
    __syncthreads();
    const float t = sh.thr_f;
    if (dense_mode) {
      // every lane of a warp takes part in each append
      for (int64_t e0 = 0; e0 < s.head_n; e0 += NT) {
        const int64_t e = e0 + tid;
        const float x = (e < s.head_n) ? Elem<T>::ld(row + e) : -INFINITY;
        if (!append_dense(!row_ovf && e < s.head_n && x >= t, x, (uint32_t)e, candB, &sh.app_n)) ovf = true;
      }
      for (int64_t e0 = 0; e0 < s.tail_n; e0 += NT) {
        const int64_t e = e0 + tid;
        const float x = (e < s.tail_n) ? Elem<T>::ld(row + s.tail_e0 + e) : -INFINITY;
        if (!append_dense(!row_ovf && e < s.tail_n && x >= t, x, (uint32_t)(s.tail_e0 + e), candB, &sh.app_n))
          ovf = true;
      }
    } else {
      for (int64_t e = tid; e < s.head_n; e += NT) {
        const float x = Elem<T>::ld(row + e);
        if (x >= t) push(x, (uint32_t)e);
      }
      for (int64_t e = tid; e < s.tail_n; e += NT) {
        const float x = Elem<T>::ld(row + s.tail_e0 + e);
        if (x >= t) push(x, (uint32_t)(s.tail_e0 + e));
      }
    }
    if (__syncthreads_or(ovf)) row_ovf = true;
    if (!row_ovf) {
      if (dense_mode) nc = dense_slots(sh.app_n);
      // shrink the list to this slice's top_k (plus ties), then pack it densely into the idle ring
      compact(top_k);
      uint32_t tot;
      const uint32_t pos = block_excl_scan<uint32_t, NT>((uint32_t)nc, sh.s32, &tot);
      uint64_t* dense = reinterpret_cast<uint64_t*>(regA);
      for (int j = 0; j < nc; ++j) dense[pos + j] = candB[j * NT + tid];
      if (tid == 0) sh.cand_n = (int32_t)tot;
    }
    if (tid == 0) sh.overflow = row_ovf ? 1 : 0;
  }

  // CTA reduction: (first maximum, its index), NaN-propagating max, smallest value above -inf
  {
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xFFFFFFFFu, bestv, o);
      const uint32_t i2 = __shfl_xor_sync(0xFFFFFFFFu, bidx, o);
      if (v2 > bestv || (v2 == bestv && i2 < bidx)) {
        bestv = v2;
        bidx = i2;
      }
      runmax = fmax_nan(runmax, __shfl_xor_sync(0xFFFFFFFFu, runmax, o));
      mnv = fminf(mnv, __shfl_xor_sync(0xFFFFFFFFu, mnv, o));
    }
    __shared__ float wf[NW], wmx[NW], wmn[NW];
    __shared__ uint32_t wi[NW];
    if ((tid & 31) == 0) {
      wf[tid >> 5] = bestv;
      wi[tid >> 5] = bidx;
      wmx[tid >> 5] = runmax;
      wmn[tid >> 5] = mnv;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < NW; ++w) {
        if (wf[w] > bestv || (wf[w] == bestv && wi[w] < bidx)) {
          bestv = wf[w];
          bidx = wi[w];
        }
        runmax = fmax_nan(runmax, wmx[w]);
        mnv = fminf(mnv, wmn[w]);
      }
      sh.pub_best = bestv;
      sh.pub_max = runmax;
      sh.pub_idx = bidx;
      sh.pub_mnv = mnv;
      sh.pub_cand_n = (filtering && !sh.overflow) ? sh.cand_n : 0;
      sh.pub_overflow = sh.overflow;
      sh.pub_timeout = sh.timeout;
    }
  }
  csync();  // S1: stage-1 results visible cluster-wide

  if (tid == 0) {
    float bv = -INFINITY, rm = -INFINITY, mn = INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    int ov = 0, to = 0;
    for (int r = 0; r < C; ++r) {
      const Shared* p = cluster.map_shared_rank(&sh, r);
      if (p->pub_best > bv || (p->pub_best == bv && p->pub_idx < bi)) {
        bv = p->pub_best;
        bi = p->pub_idx;
      }
      rm = fmax_nan(rm, p->pub_max);
      mn = fminf(mn, p->pub_mnv);
      ov |= p->pub_overflow;
      to |= p->pub_timeout;
    }
    sh.row_best = bv;
    sh.row_max = rm;
    sh.row_mnv = mn;
    sh.arg = (bi == 0xFFFFFFFFu) ? 0u : bi;  // every value -inf: the first index
    sh.any_overflow = ov;
    sh.any_timeout = to;
  }
  __syncthreads();

  // scaled extremes: x / T is monotone, so the extreme raw values give the extreme keys
  const float m = greedy ? sh.row_max : __fdiv_rn(sh.row_max, tf);
  const uint32_t mk = key_of(m);
  float* prow = a.out_probs ? a.out_probs + item * V : nullptr;
  pb_row_info info = {};
  info.max_key = (greedy && sh.row_max == sh.row_max) ? sh.row_best : m;
  int64_t token = -1;
  bool finished = false;
  pb_cand_header cand_hdr = {0, PB_CAND_FALLBACK, 0.0f, 0};  // shard mode: what this row publishes

  auto zero_probs = [&]() {
    if (prow)
      for (int64_t e = s.e_lo + tid; e < s.e_hi; e += NT) prow[e] = 0.0f;
  };

  if (sh.any_timeout) {
    info.status = PB_ROW_TIMEOUT;
    finished = true;
  } else if (sh.status != PB_ROW_OK) {
    info.status = sh.status;
    info.max_key = 0.0f;
    finished = true;
  } else if (greedy) {
    if (sh.row_max != sh.row_max) {
      // NaN in the row: torch.argmax returns the first NaN
      if (tid == 0) sh.nan_idx = 0xFFFFFFFFu;
      __syncthreads();
      for_slice<T>(row, s, [&](float x, uint32_t e) {
        if (x != x) atomicMin(&sh.nan_idx, e);
      });
      __syncthreads();
      csync();
      if (tid == 0) {
        uint32_t ni = 0xFFFFFFFFu;
        for (int r = 0; r < C; ++r) ni = min(ni, cluster.map_shared_rank(&sh, r)->nan_idx);
        sh.arg = ni;
      }
      __syncthreads();
    }
    token = sh.arg;
    info.thr_key = key_of(info.max_key);
    info.n_tie_kept = 1;
    info.kept_count = 1;
    info.flags = PB_PATH_GREEDY;
    zero_probs();
    csync();
    if (prow && rank == 0 && tid == 0) prow[token] = 1.0f;
    finished = true;
  } else if (mk >= KEY_POS_INF || mk <= KEY_NEG_INF) {
    // a shard whose values are all -inf cannot tell whether the whole row is: it defers
    if (!(a.cand_out && mk <= KEY_NEG_INF)) info.status = PB_ROW_NONFINITE;
    finished = true;
  } else if (!sh.draw_ok) {
    info.status = PB_ROW_BAD_UNIFORM;
    finished = true;
  }

  const bool topp_active = sh.top_p < 1.0 && (float)sh.top_p < 1.0f;
  const float pf = (float)sh.top_p;
  const uint64_t u53 = sh.u53;

  // ---------------- small path: survivors resolved in rank 0 ----------------
  if (!finished && filtering && !sh.any_overflow) {
    uint64_t* K = reinterpret_cast<uint64_t*>(regA + NBIN * 24);
    zero_probs();
    if (rank == 0) {
      // concatenate the CTAs' packed lists (rank r's list sits at the start of its ring)
      int32_t counts[8], offs[8];
      int32_t total = 0;
      for (int r = 0; r < C; ++r) {
        counts[r] = cluster.map_shared_rank(&sh, r)->pub_cand_n;
        offs[r] = total;
        total += counts[r];
      }
      const bool fits = total > 0 && total <= CAND_CAP;
      if (fits) {
        for (int r = 0; r < C; ++r) {
          const uint64_t* L = cluster.map_shared_rank(reinterpret_cast<uint64_t*>(regA), r);
          for (int i = tid; i < counts[r]; i += NT) candB[offs[r] + i] = L[i];
        }
      }
      if (tid == 0) {
        sh.nk = fits ? 0 : KCAP + 1;
        sh.bucket_kth = 0;
      }
      __syncthreads();
      if (fits) {
        const uint32_t kq = (uint32_t)min(top_k, total);
        uint32_t kth_raw;
        if (total <= NT) {
          // exact kq-th largest raw key by counting: the key with #greater < kq <= #greater-or-equal
          // (every thread reads the same entry at a time: shared-memory broadcasts)
          const uint32_t* hk = reinterpret_cast<const uint32_t*>(candB);  // high words: the keys
          if (tid < total) {
            const uint32_t mine = hk[2 * tid + 1];
            uint32_t gt = 0, ge = 0;
            for (int i = 0; i < total; ++i) {
              const uint32_t b = hk[2 * i + 1];
              gt += (b > mine) ? 1u : 0u;
              ge += (b >= mine) ? 1u : 0u;
            }
            if (gt < kq && kq <= ge) atomicMax(&sh.bucket_kth, mine);  // the hits hold equal keys
          }
          __syncthreads();
          kth_raw = sh.bucket_kth;
        } else {
          uint32_t kk[SLOTS];
          uint32_t mn = 0xFFFFFFFFu, mx = 0;
#pragma unroll
          for (int j = 0; j < SLOTS; ++j) {
            const int i = j * NT + tid;
            kk[j] = (i < total) ? comp_key(candB[i]) : 0u;
            if (i < total) mn = min(mn, kk[j]);
            mx = max(mx, kk[j]);
          }
          uint32_t unused, kmin, kmax;
          block_sum_min_max(0u, mn, mx, sh, &unused, &kmin, &kmax);
          kth_raw = block_kth_select<SLOTS>(kk, kq, kmin, (uint32_t)total, (uint64_t)kmax + 1, true, sh);
        }
        const uint32_t kth = key_of(__fdiv_rn(value_of(kth_raw), tf));
        for (int i0 = 0; i0 < total; i0 += NT) {
          const int i = i0 + tid;
          const uint64_t c = (i < total) ? candB[i] : 0ull;
          const uint32_t k = (i < total) ? key_of(__fdiv_rn(value_of(comp_key(c)), tf)) : 0u;
          warp_append(i < total && k >= kth, k, comp_idx(c), K, &sh.nk, KCAP);
        }
      }
      __syncthreads();
      const int nk = sh.nk;
      if (a.cand_out) {
        // vocabulary-parallel shard: publish the survivors (global indices) instead of drawing
        uint8_t* rec = a.cand_out + item * record_bytes(a.cand_cap);
        uint64_t* ent = reinterpret_cast<uint64_t*>(rec + sizeof(pb_cand_header));
        const bool fits_rec = nk <= min(a.cand_cap, KCAP);
        if (fits_rec)
          for (int i = tid; i < nk; i += NT)
            ent[i] = compose(comp_key(K[i]), comp_idx(K[i]) + (uint32_t)a.vocab_offset);
        if (tid == 0) {
          cand_hdr.count = fits_rec ? nk : 0;
          cand_hdr.flags = fits_rec ? 0 : PB_CAND_FALLBACK;
          sh.found_pos = -1;
          sh.dec.action = ACT_DONE;
        }
      } else if (nk <= KCAP) {
        finish_survivors(K, nk, m, topp_active, pf, u53, sh, &token, &info);
        if (tid == 0) sh.dec.action = ACT_DONE;
      } else {
        if (tid == 0) sh.dec.action = ACT_REFINE;  // too many survivors: cooperative path
      }
      __syncthreads();
    }
    csync();  // S2: rank 0 finished (or gave up); peers' zero-fill done
    pull_dec(cluster, sh);
    if (sh.dec_local.action == ACT_DONE) {
      if (rank == 0 && prow) {
        const int last = sh.found_pos;
        const float zf = __fmul_rn(__ull2float_rn(sh.s64[NW + 1]), 0x1p-40f);
        for (int p = tid; p <= last; p += NT) {
          const float w = exp_weight(__fsub_rn(value_of(comp_key(K[p])), m));
          prow[comp_idx(K[p])] = __fdiv_rn(w, zf);
        }
      }
      finished = true;
    }
    csync();  // rank 0's gather/candidate buffers are free again
  }

  // ---------------- large path: cooperative histogram selection ----------------
  if (!finished && a.cand_out) finished = true;  // shard mode: such rows fall back to full rows
  if (!finished) {
    info.flags = PB_PATH_LARGE;
    uint64_t* G = candB;  // gather list (rank 0)
    bool failed = false;

    // One selection over the ordered set {key >= kfloor} (MASS: weight > 0 as well): find the
    // element whose inclusive prefix (count or weight) first exceeds `target`. sh.dec_local holds
    // the level-1 decision on entry and the result on exit. Every thread of every CTA calls.
    auto select = [&](int mode, uint32_t kfloor, uint64_t target, bool need_index) {
      for (int level = 0; level < 40; ++level) {
        const Dec d = sh.dec_local;
        if (d.action == ACT_DONE) break;
        if (d.action == ACT_GATHER) {
          if (rank == 0 && tid == 0) sh.g_n = 0;
          csync();
          int32_t* gn = cluster.map_shared_rank(&sh.g_n, 0);
          uint64_t* g0 = cluster.map_shared_rank(G, 0);
          for_slice<T>(row, s, [&](float x, uint32_t e) {
            const uint32_t k = key_of(scaled(x));
            if (k < d.lo || k > d.hi || k < kfloor) return;
            if (mode == MODE_MASS && weight_q(value_of(k), m) == 0) return;
            const int pos = atomicAdd(gn, 1);
            if (pos < GCAP) g0[pos] = compose(k, e);
          });
          csync();
          if (rank == 0) {
            const int n = min(sh.g_n, GCAP);
            block_sort_desc(G, n);
            list_find(G, n, mode, m, (mode == MODE_MASS) ? d.above_w : d.above_c, target, sh);
            if (tid == 0) {
              Dec r = d;
              r.action = ACT_DONE;
              const int p = sh.found_pos;
              if (p < 0 || sh.g_n > GCAP) {
                r.fail = 1;
                r.res_idx = -1;
              } else {
                const uint32_t rk = comp_key(G[p]);
                const int f = first_of_key(G, n, rk);
                int l = f;
                while (l < n && comp_key(G[l]) == rk) ++l;
                r.res_key = rk;
                r.res_idx = (int32_t)comp_idx(G[p]);
                r.res_w_at = (mode == MODE_MASS) ? weight_q(value_of(rk), m) : 1ull;
                r.res_cnt_at = (uint64_t)(l - f);
                r.res_above_c = d.above_c + (uint64_t)f;
                uint64_t aw = d.above_w;
                if (mode == MODE_MASS)
                  for (int i = 0; i < f; ++i) aw += weight_q(value_of(comp_key(G[i])), m);
                else
                  aw = r.res_above_c;
                r.res_above_w = aw;
                r.aux = (uint64_t)(p - f);  // rank of the pick inside its tie group
              }
              sh.dec = r;
            }
            __syncthreads();
          }
          csync();
          pull_dec(cluster, sh);
          continue;
        }
        if (d.action == ACT_TIE) {
          // one key holds the target and its tie group outgrows the gather buffer
          const uint64_t wq = d.res_w_at;
          const uint64_t base = (mode == MODE_MASS) ? d.above_w : d.above_c;
          const uint64_t skip = (wq > 0 && target >= base) ? (target - base) / wq : 0;
          if (rank == 0 && tid == 0) sh.g_n = -1;  // index not found yet
          if (need_index) {
            // per-CTA count of the key; slices are in index order by rank
            if (tid == 0) sh.nk = 0;
            __syncthreads();
            uint32_t cnt = 0;
            for_slice<T>(row, s, [&](float x, uint32_t) {
              if (key_of(scaled(x)) == d.lo) cnt++;
            });
            cnt = warp_sum(cnt);
            if ((tid & 31) == 0 && cnt) atomicAdd(&sh.nk, (int)cnt);
            csync();
            uint64_t before = 0;
            for (int r = 0; r < rank; ++r) before += (uint64_t)cluster.map_shared_rank(&sh, r)->nk;
            const uint64_t mine = (uint64_t)sh.nk;
            const bool here = skip >= before && skip < before + mine;
            if (here) {
              const uint32_t want = (uint32_t)(skip - before);
              int32_t* gidx = cluster.map_shared_rank(&sh.g_n, 0);
              ordered_slice<T>(
                  row, s, sh, [&](float x, uint32_t) { return key_of(scaled(x)) == d.lo; },
                  [&](float, uint32_t e, uint32_t rnk) {
                    if (rnk == want) *gidx = (int32_t)e;
                  });
            }
          }
          csync();
          if (rank == 0 && tid == 0) {
            Dec r = d;
            r.action = ACT_DONE;
            r.res_key = d.lo;
            r.res_w_at = wq;
            r.res_cnt_at = d.cnt;
            r.res_above_w = d.above_w;
            r.res_above_c = d.above_c;
            r.aux = skip;
            r.res_idx = need_index ? sh.g_n : -1;
            if (need_index && sh.g_n < 0) r.fail = 1;
            sh.dec = r;
          }
          csync();
          pull_dec(cluster, sh);
          continue;
        }
        // ACT_REFINE: histogram of the next digit inside [lo, hi]
        const int shift = d.shift;
        for (int i = tid; i < NBIN; i += NT) {
          hq[i] = 0;
          hc[i] = 0;
        }
        __syncthreads();
        for_slice<T>(row, s, [&](float x, uint32_t) {
          const uint32_t k = key_of(scaled(x));
          if (k < d.lo || k > d.hi || k < kfloor) return;
          if (mode == MODE_MASS) {
            const uint64_t wq = weight_q(value_of(k), m);
            if (wq == 0) return;
            atomicAdd(reinterpret_cast<unsigned long long*>(&hq[(d.hi - k) >> shift]), (unsigned long long)wq);
          }
          atomicAdd(&hc[(d.hi - k) >> shift], 1u);
        });
        csync();
        if (rank == 0) {
          int b;
          uint64_t aw = 0, ac = 0, bw = 0, bc = 0;
          const int nb = (int)(((uint64_t)d.hi - d.lo) >> shift) + 1;
          const uint64_t base = (mode == MODE_MASS) ? d.above_w : d.above_c;
          reduce_and_find(cluster, C, hq, hc, hq, hc, nb, mode, target - base, sh, &b, &aw, &ac, &bw, &bc);
          if (tid == 0) {
            Dec r = d;
            if (b < 0) {
              r.action = ACT_DONE;
              r.fail = 1;
              r.res_idx = -1;
            } else {
              const uint64_t nhi = (uint64_t)d.hi - ((uint64_t)b << shift);
              const int64_t nlo = max((int64_t)d.lo, (int64_t)nhi - ((int64_t)1 << shift) + 1);
              r.hi = (uint32_t)nhi;
              r.lo = (uint32_t)nlo;
              r.above_c = d.above_c + ac;
              r.above_w = (mode == MODE_MASS) ? d.above_w + aw : r.above_c;
              r.cnt = bc;
              r.w_in = bw;
              if (r.lo == r.hi && bc > GCAP) {
                r.action = ACT_TIE;
                r.res_w_at = (mode == MODE_MASS) ? weight_q(value_of(r.lo), m) : 1ull;
              } else if (bc <= GCAP) {
                r.action = ACT_GATHER;
              } else {
                r.action = ACT_REFINE;
                r.shift = max(0, (32 - __clz(r.hi - r.lo)) - 11);
              }
            }
            sh.dec = r;
          }
          __syncthreads();
        }
        csync();
        pull_dec(cluster, sh);
      }
      if (sh.dec_local.action != ACT_DONE || sh.dec_local.fail) failed = true;
    };

    // Level-1 decision from the reduced histogram h1q/h1c (rank 0 threads only). The caller
    // brackets it with cluster barriers so that no peer still reads the previous decision.
    auto level1 = [&](int mode, float scale, uint64_t target) {
      if (tid == 0) {
        Dec r = {};
        r.action = ACT_DONE;
        r.fail = 1;
        r.res_idx = -1;
        sh.dec = r;
      }
      const int per = (NBIN + NT - 1) / NT;
      const int b0 = min(NBIN, tid * per), b1 = min(NBIN, b0 + per);
      uint64_t sw = 0, sc = 0;
      for (int b = b0; b < b1; ++b) {
        sw += (mode == MODE_MASS) ? h1q[b] : (uint64_t)h1c[b];
        sc += h1c[b];
      }
      uint64_t tw, tc;
      const uint64_t ew = block_excl_scan<uint64_t, NT>(sw, sh.s64, &tw);
      const uint64_t ec = block_excl_scan<uint64_t, NT>(sc, sh.s64, &tc);
      if (ew <= target && target < ew + sw) {
        uint64_t rw = ew, rcn = ec;
        for (int b = b0; b < b1; ++b) {
          const uint64_t wb = (mode == MODE_MASS) ? h1q[b] : (uint64_t)h1c[b];
          if (rw + wb > target) {
            Dec r = {};
            bin_interval(b, mk, m, scale, &r.lo, &r.hi);
            r.above_w = rw;
            r.above_c = rcn;
            r.cnt = h1c[b];
            r.w_in = wb;
            r.res_idx = -1;
            if (r.lo == r.hi && r.cnt > GCAP) {
              r.action = ACT_TIE;
              r.res_w_at = (mode == MODE_MASS) ? weight_q(value_of(r.lo), m) : 1ull;
            } else if (r.cnt <= GCAP) {
              r.action = ACT_GATHER;
            } else {
              r.action = ACT_REFINE;
              r.shift = max(0, (32 - __clz(r.hi - r.lo)) - 11);
            }
            sh.dec = r;
            break;
          }
          rw += wb;
          rcn += h1c[b];
        }
      }
      __syncthreads();
    };

    // Local level-1 histogram over {key >= kfloor}, reduced into rank 0's h1q/h1c.
    auto level1_pass = [&](int mode, uint32_t kfloor, float scale) {
      for (int i = tid; i < NBIN; i += NT) {
        hq[i] = 0;
        hc[i] = 0;
      }
      __syncthreads();
      for_slice<T>(row, s, [&](float x, uint32_t) {
        const uint32_t k = key_of(scaled(x));
        if (k < kfloor) return;
        const float y = value_of(k);
        const int b = bin_of(y, m, scale);
        if (mode == MODE_MASS) {
          const uint64_t wq = weight_q(y, m);
          if (wq == 0) return;
          atomicAdd(reinterpret_cast<unsigned long long*>(&hq[b]), (unsigned long long)wq);
        }
        atomicAdd(&hc[b], 1u);
      });
      csync();
      if (rank == 0) {
        for (int b = tid; b < NBIN; b += NT) {
          uint64_t q = 0;
          uint32_t c = 0;
          for (int r = 0; r < C; ++r) {
            q += cluster.map_shared_rank(hq, r)[b];
            c += cluster.map_shared_rank(hc, r)[b];
          }
          h1q[b] = q;
          h1c[b] = c;
        }
        __syncthreads();
      }
    };

    const float kmin_v = (sh.row_mnv < INFINITY) ? __fdiv_rn(sh.row_mnv, tf) : m;
    const float range_all = __fsub_rn(m, kmin_v);
    // (a range below NBIN / FLT_MAX would make the scale infinite and the max's bin 0 * inf = NaN:
    // the largest finite scale keeps the bins monotone in the key)
    const float scale_all = (range_all > 0.0f) ? fminf(__fdiv_rn((float)NBIN, range_all), 0x1.fffffep127f) : 0.0f;
    const float range_mass = fminf(range_all, MASS_RANGE);
    const float scale_mass = (range_mass > 0.0f) ? fminf(__fdiv_rn((float)NBIN, range_mass), 0x1.fffffep127f) : 0.0f;

    // (a) top-k over the whole row when the streamed candidates could not settle it
    uint32_t kfloor = 0;
    const bool topk_active = top_k > 0 && (int64_t)top_k < V;
    if (topk_active) {
      level1_pass(MODE_COUNT, 0, scale_all);
      if (rank == 0) level1(MODE_COUNT, scale_all, (uint64_t)(top_k - 1));
      csync();
      pull_dec(cluster, sh);
      select(MODE_COUNT, 0, (uint64_t)(top_k - 1), false);
      kfloor = sh.dec_local.res_key;
      csync();
    }

    // (b) pass Z: weight mass by level-1 bin over the survivors K = {key >= kfloor}
    level1_pass(MODE_MASS, kfloor, scale_mass);
    if (rank == 0) {
      uint64_t sum = 0;
      for (int b = tid; b < NBIN; b += NT) sum += h1q[b];
      uint64_t tot;
      block_excl_scan<uint64_t, NT>(sum, sh.s64, &tot);
      if (tid == 0) sh.dec.aux = tot;
      __syncthreads();
    }
    csync();
    pull_dec(cluster, sh);
    const uint64_t zq = sh.dec_local.aux;
    csync();

    // (c) top-p cut: the last kept position is the element whose inclusive mass first exceeds tp
    uint32_t cut_key = 0;
    uint64_t n_keep = 0, kept = zq;
    const bool cut = topp_active && !failed;
    if (cut) {
      const uint64_t tp = mul_floor(pf, zq);
      if (rank == 0) level1(MODE_MASS, scale_mass, tp);
      csync();
      pull_dec(cluster, sh);
      select(MODE_MASS, kfloor, tp, false);
      const Dec r = sh.dec_local;
      if (!failed && r.res_w_at > 0 && tp >= r.res_above_w) {
        cut_key = r.res_key;
        const uint64_t room = (tp - r.res_above_w) / r.res_w_at + 1;
        n_keep = min(room, r.res_cnt_at);
        kept = r.res_above_w + n_keep * r.res_w_at;
      } else {
        failed = true;
      }
      csync();
    }

    // (d) the draw over the kept prefix (t < kept, so it never reaches past the cut)
    if (!failed) {
      const uint64_t t = scale_u53(u53, kept);
      if (rank == 0) level1(MODE_MASS, scale_mass, t);
      csync();
      pull_dec(cluster, sh);
      select(MODE_MASS, kfloor, t, true);
      token = sh.dec_local.res_idx;
      csync();
    }
    if (failed) info.status = PB_ROW_INTERNAL;
    info.z_q = zq;
    info.kept_q = kept;

    // (e) kept-set description and probabilities (only when asked for)
    if ((a.out_info || prow) && !failed) {
      const float zf = __fmul_rn(__ull2float_rn(kept), 0x1p-40f);
      // per-CTA count of the cut key; slices are in index order by rank
      if (tid == 0) sh.nk = 0;
      __syncthreads();
      uint32_t cnt = 0;
      if (cut)
        for_slice<T>(row, s, [&](float x, uint32_t) {
          if (key_of(scaled(x)) == cut_key) cnt++;
        });
      cnt = warp_sum(cnt);
      if ((tid & 31) == 0 && cnt) atomicAdd(&sh.nk, (int)cnt);
      csync();
      uint64_t before = 0;
      for (int r = 0; r < rank; ++r) before += (uint64_t)cluster.map_shared_rank(&sh, r)->nk;
      uint32_t kc = 0, kmin_kept = 0xFFFFFFFFu, kmin_cnt = 0;
      for_slice<T>(row, s, [&](float x, uint32_t e) {
        const uint32_t k = key_of(scaled(x));
        if (cut && k == cut_key) return;  // settled in index order below
        const bool keep = k >= kfloor && !(cut && k < cut_key);
        if (keep) {
          kc++;
          if (k < kmin_kept) {
            kmin_kept = k;
            kmin_cnt = 1;
          } else if (k == kmin_kept) {
            kmin_cnt++;
          }
        }
        if (prow) prow[e] = keep ? __fdiv_rn(exp_weight(__fsub_rn(value_of(k), m)), zf) : 0.0f;
      });
      if (cut) {
        const float pcut = __fdiv_rn(exp_weight(__fsub_rn(value_of(cut_key), m)), zf);
        ordered_slice<T>(
            row, s, sh, [&](float x, uint32_t) { return key_of(scaled(x)) == cut_key; },
            [&](float, uint32_t e, uint32_t rnk) {
              const bool keep = before + rnk < n_keep;
              if (keep) kc++;
              if (prow) prow[e] = keep ? pcut : 0.0f;
            });
      }
      kc = warp_sum(kc);
      for (int o = 16; o > 0; o >>= 1) {
        const uint32_t k2 = __shfl_xor_sync(0xFFFFFFFFu, kmin_kept, o);
        const uint32_t c2 = __shfl_xor_sync(0xFFFFFFFFu, kmin_cnt, o);
        if (k2 < kmin_kept) {
          kmin_kept = k2;
          kmin_cnt = c2;
        } else if (k2 == kmin_kept) {
          kmin_cnt += c2;
        }
      }
      __shared__ uint32_t rk[NW], rc2[NW], rkc[NW];
      if ((tid & 31) == 0) {
        rk[tid >> 5] = kmin_kept;
        rc2[tid >> 5] = kmin_cnt;
        rkc[tid >> 5] = kc;
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t K0 = 0xFFFFFFFFu, C0 = 0, T0 = 0;
        for (int w = 0; w < NW; ++w) {
          T0 += rkc[w];
          if (rk[w] < K0) {
            K0 = rk[w];
            C0 = rc2[w];
          } else if (rk[w] == K0) {
            C0 += rc2[w];
          }
        }
        sh.pub_key = K0;
        sh.pub_idx = C0;
        sh.pub_min = T0;
      }
      csync();
      if (rank == 0 && tid == 0) {
        uint32_t K0 = 0xFFFFFFFFu, C0 = 0, T0 = 0;
        for (int r = 0; r < C; ++r) {
          const Shared* p = cluster.map_shared_rank(&sh, r);
          T0 += p->pub_min;
          if (p->pub_key < K0) {
            K0 = p->pub_key;
            C0 = p->pub_idx;
          } else if (p->pub_key == K0) {
            C0 += p->pub_idx;
          }
        }
        info.kept_count = (int32_t)T0;
        info.thr_key = cut ? cut_key : K0;
        info.n_tie_kept = cut ? (int32_t)n_keep : (int32_t)C0;
      }
    }
    finished = true;
  }

  if (rank == 0 && tid == 0 && a.cand_out) {
    uint8_t* rec = a.cand_out + item * record_bytes(a.cand_cap);
    pb_cand_header* h = reinterpret_cast<pb_cand_header*>(rec);
    if (info.status != PB_ROW_OK) {
      cand_hdr.count = 0;
      cand_hdr.flags = info.status;
    } else if (greedy) {
      reinterpret_cast<uint64_t*>(rec + sizeof(pb_cand_header))[0] =
          compose(key_of(info.max_key), (uint32_t)token + (uint32_t)a.vocab_offset);
      cand_hdr.count = 1;
      cand_hdr.flags = PB_CAND_GREEDY;
    }
    h->count = cand_hdr.count;
    h->flags = cand_hdr.flags;
    h->max_key = info.max_key;
    h->reserved = 0;
  } else if (rank == 0 && tid == 0) {
    a.out_token[item] = (info.status == PB_ROW_OK) ? token : -1;
    if (a.out_info) {  // field by field: records sit at 40-byte strides
      pb_row_info* o = a.out_info + item;
      o->thr_key = info.thr_key;
      o->n_tie_kept = info.n_tie_kept;
      o->kept_count = info.kept_count;
      o->status = info.status;
      o->max_key = info.max_key;
      o->flags = info.flags;
      o->z_q = info.z_q;
      o->kept_q = info.kept_q;
    }
  }
  csync();  // no CTA leaves while another may still read its shared memory
}

// ---- vocabulary-parallel merge -----------------------------------------------------------

constexpr int MERGE_CAP = 4096;  // union entries one row's merge resolves in shared memory
constexpr int MERGE_SMEM = MERGE_CAP * 8 + KCAP * 8;

struct MergeArgs {
  const uint8_t* records;  // [n_shards][n_rows][record_bytes(cap)]
  int32_t n_shards;
  int64_t n_rows;
  int32_t cap;
  const pb_row_params* params;
  int64_t* out_token;
  pb_row_info* out_info;
  int32_t complement;  // merge only the rows the one-warp merge marked (it ran first on the stream)
};

// One CTA per row: the row's token from the union of its shards' survivors, by the same steps and
// arithmetic as the small path of sample_kernel (exact k-th key, fixed-point weights, top-p cut,
// inverse-CDF draw), so the result equals sampling the full row.
__global__ void __launch_bounds__(NT, 1) merge_kernel(MergeArgs a) {
  extern __shared__ __align__(128) unsigned char dyn[];
  __shared__ Shared sh;
  uint64_t* L = reinterpret_cast<uint64_t*>(dyn);                  // the union of the records
  uint64_t* K = reinterpret_cast<uint64_t*>(dyn + MERGE_CAP * 8);  // the row's survivors
  const int64_t item = blockIdx.x;
  const int tid = threadIdx.x;
  if (a.complement) {
    griddep_wait();
    if (a.out_token[item] != F_RETRY) return;
  }
  const int64_t rb = record_bytes(a.cap);
  auto header = [&](int r) {
    return reinterpret_cast<const pb_cand_header*>(a.records + ((int64_t)r * a.n_rows + item) * rb);
  };
  auto entries = [&](int r) { return reinterpret_cast<const uint64_t*>(header(r) + 1); };

  if (tid == 0) {
    const pb_row_params p = a.params[item];
    sh.temperature = p.temperature;
    sh.top_p = p.top_p;
    sh.u53 = row_u53(p);
    sh.draw_ok = row_draw_ok(p) ? 1 : 0;
    sh.top_k = p.top_k;
    sh.greedy = (p.temperature == 0.0);
    sh.tf = (float)p.temperature;
    int32_t fl = 0, total = 0;
    float gmax = -INFINITY;
    uint64_t best = 0;
    int best_r = 0;
    for (int r = 0; r < a.n_shards; ++r) {
      const pb_cand_header* h = header(r);
      fl |= h->flags;
      total += h->count;
      gmax = fmax_nan(gmax, h->max_key);
      if ((h->flags & PB_CAND_GREEDY) && h->count == 1 && entries(r)[0] > best) {
        best = entries(r)[0];
        best_r = r;
      }
    }
    sh.status = PB_ROW_OK;
    const bool bad = !(p.temperature >= 0.0) || !(p.top_p > 0.0 && p.top_p <= 1.0) || p.top_k < 0;
    const uint32_t mk = key_of(gmax);
    int mode = 0;  // 0 status only, 1 greedy, 2 merge
    if (fl & PB_ROW_TIMEOUT) sh.status = PB_ROW_TIMEOUT;
    else if (bad) sh.status = PB_ROW_BAD_PARAMS;
    else if (sh.greedy) mode = 1;
    else if (mk >= KEY_POS_INF || mk <= KEY_NEG_INF) sh.status = PB_ROW_NONFINITE;
    else if (!row_draw_ok(p)) sh.status = PB_ROW_BAD_UNIFORM;
    else if ((fl & (PB_CAND_FALLBACK | 0xFF)) || total > MERGE_CAP || total == 0) sh.status = PB_ROW_FALLBACK;
    else mode = 2;
    if (mode == 1 && (fl & ~PB_CAND_GREEDY)) {  // a shard could not publish its maximum
      sh.status = PB_ROW_FALLBACK;
      mode = 0;
    }
    sh.cand_n = total;
    sh.nk = mode;
    sh.row_max = gmax;
    sh.row_best = header(best_r)->max_key;
    sh.arg = comp_idx(best);
    sh.mk = key_of(gmax);
  }
  __syncthreads();
  const int mode = sh.nk;
  pb_row_info info = {};
  int64_t token = -1;
  info.status = sh.status;
  if (mode == 1) {
    info.max_key = sh.row_best;
    info.thr_key = key_of(info.max_key);
    info.n_tie_kept = 1;
    info.kept_count = 1;
    info.flags = PB_PATH_GREEDY;
    token = sh.arg;
  } else if (mode == 2) {
    const float m = sh.row_max;
    const int total = sh.cand_n;
    const int32_t top_k = sh.top_k;
    info.max_key = m;
    // gather the union (shards in order; entry order does not matter)
    int off = 0;
    for (int r = 0; r < a.n_shards; ++r) {
      const int n = header(r)->count;
      const uint64_t* e = entries(r);
      for (int i = tid; i < n; i += NT) L[off + i] = e[i];
      off += n;
    }
    __syncthreads();
    uint32_t kk[MERGE_CAP / NT];
    uint32_t mn = 0xFFFFFFFFu, mx = 0;
#pragma unroll
    for (int j = 0; j < MERGE_CAP / NT; ++j) {
      const int i = j * NT + tid;
      kk[j] = (i < total) ? comp_key(L[i]) : 0u;
      if (i < total) mn = min(mn, kk[j]);
      mx = max(mx, kk[j]);
    }
    uint32_t unused, kmin, kmax;
    block_sum_min_max(0u, mn, mx, sh, &unused, &kmin, &kmax);
    const int kq = (top_k > 0) ? min(top_k, total) : total;
    const uint32_t kth = block_kth_select<MERGE_CAP / NT>(kk, (uint32_t)kq, kmin, (uint32_t)total, (uint64_t)kmax + 1,
                                                          true, sh);
    if (tid == 0) sh.nk = 0;
    __syncthreads();
    for (int i0 = 0; i0 < total; i0 += NT) {
      const int i = i0 + tid;
      const uint64_t c = (i < total) ? L[i] : 0ull;
      warp_append(i < total && comp_key(c) >= kth, comp_key(c), comp_idx(c), K, &sh.nk, KCAP);
    }
    __syncthreads();
    const int nk = sh.nk;
    if (nk <= KCAP) {
      const bool topp_active = sh.top_p < 1.0 && (float)sh.top_p < 1.0f;
      finish_survivors(K, nk, m, topp_active, (float)sh.top_p, sh.u53, sh, &token, &info);
    } else if (tid == 0) {
      info.status = PB_ROW_FALLBACK;
    }
  } else if (sh.status == PB_ROW_NONFINITE || sh.status == PB_ROW_BAD_UNIFORM || sh.status == PB_ROW_TIMEOUT) {
    info.max_key = sh.row_max;
  }
  if (tid == 0) {
    a.out_token[item] = (info.status == PB_ROW_OK) ? token : -1;
    if (a.out_info) {
      pb_row_info* o = a.out_info + item;
      o->thr_key = info.thr_key;
      o->n_tie_kept = info.n_tie_kept;
      o->kept_count = info.kept_count;
      o->status = info.status;
      o->max_key = info.max_key;
      o->flags = info.flags;
      o->z_q = info.z_q;
      o->kept_q = info.kept_q;
    }
  }
}

// The merge with one warp per row (8 rows per CTA), by the finisher's steps: the union of the
// records, cut to the entries at or above the largest k-th key among the shards that hold at least
// k entries (a lower bound of the row's k-th key: such a shard alone holds k values at or above
// its own k-th), sorted in registers, then the k-th key, the survivors, the top-p cut and the draw.
// A row whose cut union is longer than F_LCAP is marked F_RETRY for merge_kernel.
constexpr int MW_ROWS = 8;
constexpr int MW_SMEM = MW_ROWS * F_LCAP * 8;

__global__ void __launch_bounds__(MW_ROWS * 32) merge_warp_kernel(MergeArgs m) {
  extern __shared__ __align__(16) unsigned char dyn[];
  griddep_launch_dependents();  // merge_kernel (the long rows) may launch; it waits for this grid
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const int64_t item = (int64_t)blockIdx.x * MW_ROWS + wi;
  if (item >= m.n_rows) return;  // (the whole warp; this kernel has no block-wide step)
  uint64_t* L = reinterpret_cast<uint64_t*>(dyn) + wi * F_LCAP;
  const int64_t rb = record_bytes(m.cap);
  auto hdr = [&](int r) {
    return reinterpret_cast<const pb_cand_header*>(m.records + ((int64_t)r * m.n_rows + item) * rb);
  };
  auto ent = [&](int r) { return reinterpret_cast<const uint64_t*>(hdr(r) + 1); };
  const pb_row_params p = m.params[item];
  int32_t fl = 0, total = 0;
  float gmax = -INFINITY, bmk = 0.0f;
  uint64_t best = 0;
  for (int r = lane; r < m.n_shards; r += 32) {
    const pb_cand_header h = *hdr(r);
    fl |= h.flags;
    total += h.count;
    gmax = fmax_nan(gmax, h.max_key);
    if ((h.flags & PB_CAND_GREEDY) && h.count == 1) {
      const uint64_t e = ent(r)[0];
      if (e > best) {
        best = e;
        bmk = h.max_key;
      }
    }
  }
  fl = (int32_t)__reduce_or_sync(0xFFFFFFFFu, (uint32_t)fl);
  total = (int32_t)__reduce_add_sync(0xFFFFFFFFu, (uint32_t)total);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    gmax = fmax_nan(gmax, __shfl_xor_sync(0xFFFFFFFFu, gmax, o));
    const uint64_t b2 = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const float m2 = __shfl_xor_sync(0xFFFFFFFFu, bmk, o);
    if (b2 > best) {
      best = b2;
      bmk = m2;
    }
  }
  const bool bad = !(p.temperature >= 0.0) || !(p.top_p > 0.0 && p.top_p <= 1.0) || p.top_k < 0;
  const uint32_t mk = key_of(gmax);
  int mode = 0, status = PB_ROW_OK;  // mode 0 status only, 1 greedy, 2 merge
  if (fl & PB_ROW_TIMEOUT) status = PB_ROW_TIMEOUT;
  else if (bad) status = PB_ROW_BAD_PARAMS;
  else if (p.temperature == 0.0) mode = 1;
  else if (mk >= KEY_POS_INF || mk <= KEY_NEG_INF) status = PB_ROW_NONFINITE;
  else if (!row_draw_ok(p)) status = PB_ROW_BAD_UNIFORM;
  else if ((fl & (PB_CAND_FALLBACK | 0xFF)) || total > MERGE_CAP || total == 0) status = PB_ROW_FALLBACK;
  else mode = 2;
  if (mode == 1 && (fl & ~PB_CAND_GREEDY)) {  // a shard could not publish its maximum
    status = PB_ROW_FALLBACK;
    mode = 0;
  }
  if (mode == 2) {
    const int kq = (p.top_k > 0) ? min(p.top_k, total) : total;
    uint32_t lb = 0;
    for (int r = 0; r < m.n_shards; ++r) {
      const int cnt = hdr(r)->count;
      if (cnt >= kq) {
        uint32_t mn = 0xFFFFFFFFu;
        for (int i = lane; i < cnt; i += 32) mn = min(mn, comp_key(ent(r)[i]));
        lb = max(lb, __reduce_min_sync(0xFFFFFFFFu, mn));
      }
    }
    int n = 0;
    for (int r = 0; r < m.n_shards; ++r) {
      const int cnt = hdr(r)->count;
      const uint64_t* e = ent(r);
      for (int i0 = 0; i0 < cnt; i0 += 32) {
        const int i = i0 + lane;
        const uint64_t v = (i < cnt) ? e[i] : 0ull;
        const bool keep = i < cnt && comp_key(v) >= lb;
        const uint32_t bl = __ballot_sync(0xFFFFFFFFu, keep);
        const int at = n + __popc(bl & lanemask_lt());
        if (keep && at < F_LCAP) L[at] = v;
        n += __popc(bl);
      }
    }
    __syncwarp();
    FastArgs fa = {};
    fa.out_token = m.out_token;
    fa.out_info = m.out_info;
    if (n > F_SMAX && n <= F_LCAP) {
      // cut to the survivors first: the exact kq-th key by bisection, keys at or above it
      constexpr int R = F_LCAP / 32;
      uint64_t c[R];
      uint32_t lo = 0xFFFFFFFFu, mx = 0;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const int i = j * 32 + lane;
        c[j] = (i < n) ? L[i] : 0ull;
        if (i < n) lo = min(lo, comp_key(c[j]));
        mx = max(mx, comp_key(c[j]));
      }
      lo = __reduce_min_sync(0xFFFFFFFFu, lo);
      uint64_t hi = (uint64_t)__reduce_max_sync(0xFFFFFFFFu, mx) + 1;
      const int kk = min(p.top_k, n);
      while (hi - lo > 1) {
        const uint32_t mid = (uint32_t)(lo + ((hi - lo) >> 1));
        uint32_t cnt = 0;
#pragma unroll
        for (int j = 0; j < R; ++j) cnt += (j * 32 + lane < n && comp_key(c[j]) >= mid) ? 1u : 0u;
        if ((int)__reduce_add_sync(0xFFFFFFFFu, cnt) >= kk) lo = mid;
        else hi = mid;
      }
      int w = 0;
#pragma unroll
      for (int j = 0; j < R; ++j) {
        const bool keep = j * 32 + lane < n && comp_key(c[j]) >= lo;
        const uint32_t bl = __ballot_sync(0xFFFFFFFFu, keep);
        if (keep) L[w + __popc(bl & lanemask_lt())] = c[j];
        w += __popc(bl);
      }
      __syncwarp();
      n = w;
    }
    if (n > F_SMAX) {
      if (lane == 0) m.out_token[item] = F_RETRY;  // merge_kernel takes this row
    } else if (n <= 64) {
      finish_list<2, true>(fa, p, item, L, n, gmax, PB_PATH_SMALL);
    } else if (n <= 128) {
      finish_list<4, true>(fa, p, item, L, n, gmax, PB_PATH_SMALL);
    } else {
      finish_list<8, true>(fa, p, item, L, n, gmax, PB_PATH_SMALL);
    }
    return;
  }
  if (lane == 0) {
    int64_t token = -1;
    pb_row_info info = {};
    info.status = status;
    if (mode == 1) {
      info.max_key = bmk;
      info.thr_key = key_of(bmk);
      info.n_tie_kept = 1;
      info.kept_count = 1;
      info.flags = PB_PATH_GREEDY;
      token = comp_idx(best);
    } else if (status == PB_ROW_NONFINITE || status == PB_ROW_BAD_UNIFORM || status == PB_ROW_TIMEOUT) {
      info.max_key = gmax;
    }
    m.out_token[item] = (info.status == PB_ROW_OK) ? token : -1;
    if (m.out_info) m.out_info[item] = info;
  }
}

// ---- finish reasons (pb_stop_check) ------------------------------------------------------------

// One thread per row: pagedbatch/engine.py:173-182 (_finish_reason) on the token just sampled.
__global__ void __launch_bounds__(256) stop_check_kernel(const int64_t* tokens, int64_t n_rows, const int4* state,
                                                         const int32_t* offs, const int32_t* ids, int32_t eos,
                                                         int32_t max_model_len, int8_t* out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_rows) return;
  const int64_t tok = tokens[r];
  const int4 st = state[r];  // ignore_eos, output length, max_tokens, total length
  int8_t reason = PB_FINISH_NONE;
  if (tok >= 0) {
    bool stop = false;
    if (!st.x) {
      stop = eos >= 0 && tok == eos;
      for (int32_t i = offs[r]; !stop && i < offs[r + 1]; ++i) stop = tok == ids[i];
    }
    if (stop) reason = PB_FINISH_STOP;
    else if (st.y >= st.z || st.w >= max_model_len) reason = PB_FINISH_LENGTH;
  }
  out[r] = reason;
}

// Per-device one-time set-up (a function attribute, a device property): a bit per device, set
// atomically, so that concurrent first calls from several host threads are safe (the set-up itself
// is idempotent).
struct DeviceOnce {
  std::atomic<unsigned long long> done{0};
  bool test(int dev) const { return (done.load(std::memory_order_acquire) >> dev) & 1ull; }
  void set(int dev) { done.fetch_or(1ull << dev, std::memory_order_acq_rel); }
};

int current_device(int* dev) {
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0 || *dev >= 64) return PB_E_DEVICE;
  return PB_OK;
}

// Per-device cached integer (0 = not yet known).
struct DeviceInt {
  std::atomic<int> v[64] = {};
};

int sm_count() {
  static DeviceInt cache;
  int dev = 0;
  if (current_device(&dev) != PB_OK) dev = 0;
  int n = cache.v[dev].load(std::memory_order_relaxed);
  if (!n) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache.v[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T>
int launch(const Args& a, int C, cudaStream_t stream, bool pdl = false) {
  // the dynamic shared memory limit is a per-device function attribute
  static DeviceOnce configured;
  int dev = 0;
  if (current_device(&dev) != PB_OK) return PB_E_DEVICE;
  if (!configured.test(dev)) {
    if (cudaFuncSetAttribute(sample_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, DYN_SMEM) != cudaSuccess)
      return PB_E_DEVICE;
    configured.set(dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.n_rows * C), 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = DYN_SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // after the streaming kernel: launch early, the CTAs that need its results wait for it
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, sample_kernel<T>, a) != cudaSuccess) return PB_E_LAUNCH;
  if (cudaGetLastError() != cudaSuccess) return PB_E_LAUNCH;
  return PB_OK;
}

// The persistent streaming kernel: one CTA per SM (at most one per row).
template <typename T>
int launch_stream(const FastArgs& a, int64_t grid, cudaStream_t stream) {
  static DeviceOnce configured;
  int dev = 0;
  if (current_device(&dev) != PB_OK) return PB_E_DEVICE;
  if (!configured.test(dev)) {
    if (cudaFuncSetAttribute(stream_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, F_SMEM) != cudaSuccess)
      return PB_E_DEVICE;
    configured.set(dev);
  }
  stream_kernel<T><<<(unsigned)grid, F_THREADS, F_SMEM, stream>>>(a);
  if (cudaGetLastError() != cudaSuccess) return PB_E_LAUNCH;
  return PB_OK;
}

// Cluster size: enough CTAs to give every SM one, but slices of at least one staged chunk (a
// slice shorter than a chunk pays the per-CTA start and finish for less than one ring stage).
int cluster_size_for(int64_t n_rows, int64_t vocab, int es) {
  const char* env = getenv("PB_CLUSTER");
  if (env) {
    const int c = atoi(env);
    if (c == 1 || c == 2 || c == 4 || c == 8) return c;
  }
  const int64_t want = sm_count();
  const int64_t bytes = vocab * es;
  int C = 1;
  while (C < 8 && n_rows * C < want && bytes / (2 * C) >= CHUNK_BYTES) C <<= 1;
  return C;
}

int launch_merge(const uint8_t* records, int32_t n_shards, int64_t n_rows, int32_t cap, const pb_row_params* params,
                 int64_t* out_token, pb_row_info* out_info, cudaStream_t stream) {
  static DeviceOnce configured;
  int dev = 0;
  if (current_device(&dev) != PB_OK) return PB_E_DEVICE;
  if (!configured.test(dev)) {
    if (cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MERGE_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(merge_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, MW_SMEM) != cudaSuccess)
      return PB_E_DEVICE;
    configured.set(dev);
  }
  MergeArgs m;
  m.records = records;
  m.n_shards = n_shards;
  m.n_rows = n_rows;
  m.cap = cap;
  m.params = params;
  m.out_token = out_token;
  m.out_info = out_info;
  m.complement = 0;
  merge_warp_kernel<<<(unsigned)((n_rows + MW_ROWS - 1) / MW_ROWS), MW_ROWS * 32, MW_SMEM, stream>>>(m);
  if (cudaGetLastError() != cudaSuccess) return PB_E_LAUNCH;
  m.complement = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_rows, 1, 1);
  cfg.blockDim = dim3(NT, 1, 1);
  cfg.dynamicSmemBytes = MERGE_SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, merge_kernel, m) != cudaSuccess) return PB_E_LAUNCH;
  if (cudaGetLastError() != cudaSuccess) return PB_E_LAUNCH;
  return PB_OK;
}

constexpr int64_t align256(int64_t n) { return (n + 255) & ~(int64_t)255; }

int stage_poll_limit();

// Balanced streaming launch (the workspace path): CTAs, at most one per SM, each share at least
// SEG_MIN vectors long (so no share is empty).
// PB_BALANCED_GRID caps the grid (tests use it to vary how rows are cut into pieces).
int64_t balanced_grid(int64_t n_rows, int64_t vocab, int es) {
  const int64_t epv = 16 / es;
  const int64_t N = n_rows * ((vocab + epv - 1) / epv);
  int64_t g = std::min<int64_t>((int64_t)F_CPS * sm_count(), N / SEG_MIN);
  if (const char* env = getenv("PB_BALANCED_GRID")) {
    const int64_t cap = atoll(env);
    if (cap >= 1) g = std::min(g, cap);
  }
  return std::max<int64_t>(1, g);
}

// workspace of the balanced launch: per-row arrival counters, then one record per piece (a piece is
// indexed by row + CTA, so n_rows + grid records cover every piece)
int64_t ws_need(int64_t n_rows, int64_t grid) {
  return align256(n_rows * 8) + (n_rows + grid) * record_bytes(F_SREC);
}

// balanced streaming kernel -> cluster kernel over the rows it did not take or could not settle
template <typename T>
int run_balanced(const Args& a, uint8_t* workspace, int64_t grid, int es, cudaStream_t st) {
  FastArgs f;
  f.logits = a.logits;
  f.n_rows = a.n_rows;
  f.vocab = a.vocab;
  f.row_stride = a.row_stride;
  f.row_index = a.row_index;
  f.params = a.params;
  f.out_token = a.out_token;
  f.out_info = a.out_info;
  f.cand_out = nullptr;
  f.cand_cap = 0;
  f.vocab_offset = 0;
  f.poll_limit = stage_poll_limit();
  f.balanced = 1;
  f.row_cnt = reinterpret_cast<unsigned long long*>(workspace);
  f.seg_rec = workspace + align256(a.n_rows * 8);
  int rc = launch_stream<T>(f, grid, st);
  if (rc != PB_OK) return rc;
  Args c = a;
  c.complement = 1;
  return launch<T>(c, cluster_size_for(a.n_rows, a.vocab, es), st, getenv("PB_NO_PDL") == nullptr);
}

int run_ws(const void* logits, int dtype, int es, int64_t n_rows, int64_t vocab, int64_t row_stride,
           const int32_t* row_index, const pb_row_params* params, int64_t* out_token, pb_row_info* out_info,
           uint8_t* workspace, int64_t grid, cudaStream_t st) {
  Args a;
  a.logits = static_cast<const char*>(logits);
  a.n_rows = n_rows;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.row_index = row_index;
  a.params = params;
  a.out_token = out_token;
  a.out_info = out_info;
  a.out_probs = nullptr;
  a.only_fallback = nullptr;
  a.complement = 0;
  a.cand_out = nullptr;
  a.cand_cap = 0;
  a.vocab_offset = 0;
  if (dtype == PB_DTYPE_F32) return run_balanced<float>(a, workspace, grid, es, st);
  if (dtype == PB_DTYPE_BF16) return run_balanced<__nv_bfloat16>(a, workspace, grid, es, st);
  return run_balanced<__half>(a, workspace, grid, es, st);
}

// ---- two-pass workspace path (pb_groups.cuh) ---------------------------------------------------

// Its geometry for a batch: group keys per row (and their row stride), pass-1 tasks, pass-2
// coarsening, workspace bytes.
struct GroupPlan {
  int64_t ngr, ngs, ntasks, coarse, bytes;
};

GroupPlan group_plan(int64_t n_rows, int64_t vocab, int es) {
  GroupPlan g;
  const int64_t ge = GM_GB / es;
  g.ngr = (vocab + ge - 1) / ge;
  g.ngs = (g.ngr + 3) & ~(int64_t)3;
  g.ntasks = (n_rows * g.ngr + 3) / 4;
  g.coarse = (g.ngr + GS_MAXG - 1) / GS_MAXG;
  g.bytes = align256(n_rows * g.ngs * 4);
  return g;
}

// Rows the two-pass path can read: every row starts on a 16-byte boundary (its passes load whole
// 16-byte vectors from a row's start) and the batch has fewer than 2^31 groups. PB_WS=balanced
// selects the balanced streaming launch instead.
bool groups_eligible(const void* logits, int64_t row_stride, int es, int64_t n_rows, int64_t vocab) {
  const char* env = getenv("PB_WS");
  if (env && strcmp(env, "balanced") == 0) return false;
  if (n_rows * group_plan(1, vocab, es).ngs >= (int64_t)0x7FFFFFFF) return false;
  return (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && ((row_stride * es) & 15) == 0;
}

// Pass-1 grid: GM_TPW tasks per warp, or (GM_TPW = 0) the CTAs that fit on the device at once (at
// least one task per warp).
template <typename T>
int64_t group_grid(int64_t ntasks) {
  static DeviceInt occ;
  int dev = 0;
  if (current_device(&dev) != PB_OK) dev = 0;
  int per_sm = occ.v[dev].load(std::memory_order_relaxed);
  if (!per_sm) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, group_max_kernel<T>, GM_THREADS, 0) != cudaSuccess ||
        per_sm <= 0)
      per_sm = GM_MINB;
    occ.v[dev].store(per_sm, std::memory_order_relaxed);
  }
  const int64_t full = (int64_t)per_sm * sm_count();
  if (GM_TPW > 0) return std::max<int64_t>(1, (ntasks + (int64_t)GM_TPW * GM_WARPS - 1) / ((int64_t)GM_TPW * GM_WARPS));
  return std::max<int64_t>(1, std::min<int64_t>(full, (ntasks + GM_WARPS - 1) / GM_WARPS));
}

// pass 1 -> pass 2 (programmatic dependency) -> cluster kernel over the rows pass 2 left
template <typename T>
int run_groups(const Args& a, uint8_t* workspace, int es, cudaStream_t st) {
  const GroupPlan gp = group_plan(a.n_rows, a.vocab, es);
  GroupArgs g;
  g.logits = a.logits;
  g.n_rows = a.n_rows;
  g.vocab = a.vocab;
  g.row_stride_bytes = a.row_stride * es;
  g.row_index = a.row_index;
  g.params = a.params;
  g.out_token = a.out_token;
  g.out_info = a.out_info;
  g.gmax = reinterpret_cast<uint32_t*>(workspace);
  g.ngr = (int32_t)gp.ngr;
  g.ngs = (int32_t)gp.ngs;
  g.coarse = (int32_t)gp.coarse;
  g.ntasks = gp.ntasks;
  g.cand_out = a.cand_out;
  g.cand_cap = a.cand_cap;
  g.vocab_offset = a.vocab_offset;
  group_max_kernel<T><<<(unsigned)group_grid<T>(gp.ntasks), GM_THREADS, 0, st>>>(g);
  if (cudaGetLastError() != cudaSuccess) return PB_E_LAUNCH;
  const bool pdl = getenv("PB_NO_PDL") == nullptr;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.n_rows, 1, 1);
  cfg.blockDim = dim3(GS_THREADS, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = (a.n_rows <= 2 * (int64_t)sm_count()) ? cudaLaunchKernelEx(&cfg, group_settle_kernel<T, 2>, g)
                                                              : cudaLaunchKernelEx(&cfg, group_settle_kernel<T, 4>, g);
  if (e != cudaSuccess) return PB_E_LAUNCH;
  if (cudaGetLastError() != cudaSuccess) return PB_E_LAUNCH;
  Args c = a;
  c.complement = 1;
  return launch<T>(c, cluster_size_for(a.n_rows, a.vocab, es), st, pdl);
}

int run_groups_args(const Args& a, int dtype, int es, uint8_t* workspace, cudaStream_t st) {
  if (dtype == PB_DTYPE_F32) return run_groups<float>(a, workspace, es, st);
  if (dtype == PB_DTYPE_BF16) return run_groups<__nv_bfloat16>(a, workspace, es, st);
  return run_groups<__half>(a, workspace, es, st);
}

int run_groups_dtype(const void* logits, int dtype, int es, int64_t n_rows, int64_t vocab, int64_t row_stride,
                     const int32_t* row_index, const pb_row_params* params, int64_t* out_token,
                     pb_row_info* out_info, uint8_t* workspace, cudaStream_t st) {
  Args a;
  a.logits = static_cast<const char*>(logits);
  a.n_rows = n_rows;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.row_index = row_index;
  a.params = params;
  a.out_token = out_token;
  a.out_info = out_info;
  a.out_probs = nullptr;
  a.only_fallback = nullptr;
  a.complement = 0;
  a.cand_out = nullptr;
  a.cand_cap = 0;
  a.vocab_offset = 0;
  return run_groups_args(a, dtype, es, workspace, st);
}

// ---- allocation-free entry point -------------------------------------------------------------
// Some callers cannot allocate device memory at all: plugins whose host application owns every
// byte of the GPU through its own allocator, or C callers with no allocator of their own. For
// them pb_sample_noalloc runs the workspace path with this fixed array as its workspace. Every GPU
// that loads this library holds the array until the process exits.
constexpr int64_t NOALLOC_SCRATCH_BYTES = 32ll << 20;  // 32 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device, looked up once per device (in host
// code the array's name is only a host-side stand-in, never a device address).
// The cached address stays valid for the process's primary context on that device; a caller that
// resets the device (cudaDeviceReset) must not use this entry point again in the same process.
int noalloc_scratch(uint8_t** out) {
  static std::atomic<uint8_t*> addr[64] = {};
  int dev = 0;
  if (current_device(&dev) != PB_OK) return PB_E_DEVICE;
  uint8_t* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return PB_E_DEVICE;
    a = static_cast<uint8_t*>(p);
    addr[dev].store(a, std::memory_order_release);
  }
  *out = a;
  return PB_OK;
}
// Which kernels pb_sample / pb_candidates run. The persistent streaming kernel (greedy rows and
// top_k <= F_KMAX, then the cluster kernel on the same stream over every other row and the rows it
// marked) pays off when each SM has several rows to pipeline: measured on a B200, [1024, 128256]
// bf16 rows take 99 us instead of 193 us, while [256, 128256] fp32 (1.7 rows per SM) is faster on
// the cluster kernel alone (41 us against 46 us). PB_PATH=cluster / PB_PATH=stream force one.
bool stream_path_enabled(int64_t n_rows) {
  const char* env = getenv("PB_PATH");
  if (env && strcmp(env, "cluster") == 0) return false;
  if (env && strcmp(env, "stream") == 0) return true;
  return n_rows >= 3 * (int64_t)sm_count();
}

// Consumer waits of the streaming kernel: WAIT_POLLS polls, or PB_TEST_STAGE_POLLS (a test of the
// bounded-wait path sets 0, so that every wait on a staged chunk gives up at once).
int stage_poll_limit() {
  const char* env = getenv("PB_TEST_STAGE_POLLS");
  if (env) {
    const int v = atoi(env);
    if (v >= 0 && v <= WAIT_POLLS) return v;
  }
  return WAIT_POLLS;
}

template <typename T>
int run_rows(Args a, int es, cudaStream_t st) {
  const int C = cluster_size_for(a.n_rows, a.vocab, es);
  if (a.out_probs || !stream_path_enabled(a.n_rows)) {
    a.complement = 0;
    return launch<T>(a, C, st);
  }
  FastArgs f;
  f.logits = a.logits;
  f.n_rows = a.n_rows;
  f.vocab = a.vocab;
  f.row_stride = a.row_stride;
  f.row_index = a.row_index;
  f.params = a.params;
  f.out_token = a.out_token;
  f.out_info = a.out_info;
  f.cand_out = a.cand_out;
  f.cand_cap = a.cand_cap;
  f.vocab_offset = a.vocab_offset;
  f.poll_limit = stage_poll_limit();
  f.balanced = 0;
  f.row_cnt = nullptr;
  f.seg_rec = nullptr;
  int rc = launch_stream<T>(f, std::min<int64_t>(a.n_rows, (int64_t)F_CPS * sm_count()), st);
  if (rc != PB_OK) return rc;
  a.complement = 1;
  return launch<T>(a, C, st, getenv("PB_NO_PDL") == nullptr);
}

int run_rows_dtype(const Args& a, int dtype, int es, cudaStream_t st) {
  if (dtype == PB_DTYPE_F32) return run_rows<float>(a, es, st);
  if (dtype == PB_DTYPE_BF16) return run_rows<__nv_bfloat16>(a, es, st);
  return run_rows<__half>(a, es, st);
}
}  // namespace

extern "C" {

int pb_sample(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
              const int32_t* row_index, const pb_row_params* params, int64_t* out_token, pb_row_info* out_info,
              float* out_probs, void* stream) {
  if (n_rows < 0 || vocab <= 0 || row_stride < vocab) return PB_E_INVALID;
  if (vocab >= PB_MAX_VOCAB) return PB_E_TOO_LARGE;
  if (n_rows == 0) return PB_OK;
  if (!logits || !params || !out_token) return PB_E_INVALID;
  if (n_rows > (int64_t)(0x7FFFFFFF / 8)) return PB_E_INVALID;
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(logits) % es) != 0) return PB_E_INVALID;
  Args a;
  a.logits = static_cast<const char*>(logits);
  a.n_rows = n_rows;
  a.vocab = vocab;
  a.row_stride = row_stride;
  a.row_index = row_index;
  a.params = params;
  a.out_token = out_token;
  a.out_info = out_info;
  a.out_probs = out_probs;
  a.only_fallback = nullptr;
  a.complement = 0;
  a.cand_out = nullptr;
  a.cand_cap = 0;
  a.vocab_offset = 0;
  return run_rows_dtype(a, dtype, es, static_cast<cudaStream_t>(stream));
}

int64_t pb_record_bytes(int32_t cap) { return record_bytes(cap); }

int pb_sample_ws_launches(const void* logits, int64_t n_rows, int64_t vocab, int64_t row_stride, int dtype) {
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es || n_rows < 0 || vocab <= 0) return PB_E_INVALID;
  if (n_rows == 0) return 0;
  return groups_eligible(logits, row_stride, es, n_rows, vocab) ? 3 : 2;
}

int pb_sample_launches(int64_t n_rows, int64_t vocab, int dtype, int with_probs) {
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es || n_rows < 0 || vocab <= 0) return PB_E_INVALID;
  if (n_rows == 0) return 0;
  return (!with_probs && stream_path_enabled(n_rows)) ? 2 : 1;
}

int pb_candidates(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab, int64_t row_stride,
                  const int32_t* row_index, const pb_row_params* params, int64_t vocab_offset, int32_t cap,
                  void* out_records, void* stream) {
  if (n_rows < 0 || shard_vocab <= 0 || row_stride < shard_vocab || vocab_offset < 0) return PB_E_INVALID;
  if (cap < 1 || cap > PB_CAND_MAX_CAP) return PB_E_INVALID;
  if (vocab_offset + shard_vocab >= PB_MAX_VOCAB) return PB_E_TOO_LARGE;
  if (n_rows == 0) return PB_OK;
  if (!logits || !params || !out_records) return PB_E_INVALID;
  if (n_rows > (int64_t)(0x7FFFFFFF / 8)) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(out_records) & 15) != 0) return PB_E_INVALID;
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(logits) % es) != 0) return PB_E_INVALID;
  Args a;
  a.logits = static_cast<const char*>(logits);
  a.n_rows = n_rows;
  a.vocab = shard_vocab;
  a.row_stride = row_stride;
  a.row_index = row_index;
  a.params = params;
  a.out_token = nullptr;
  a.out_info = nullptr;
  a.out_probs = nullptr;
  a.only_fallback = nullptr;
  a.complement = 0;
  a.cand_out = static_cast<uint8_t*>(out_records);
  a.cand_cap = cap;
  a.vocab_offset = vocab_offset;
  return run_rows_dtype(a, dtype, es, static_cast<cudaStream_t>(stream));
}

int64_t pb_candidates_ws_bytes(int64_t n_rows, int64_t shard_vocab, int dtype) {
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es || n_rows < 0 || shard_vocab <= 0) return PB_E_INVALID;
  return group_plan(n_rows, shard_vocab, es).bytes;
}

int pb_candidates_ws(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab, int64_t row_stride,
                     const int32_t* row_index, const pb_row_params* params, int64_t vocab_offset, int32_t cap,
                     void* out_records, void* workspace, int64_t ws_bytes, void* stream) {
  if (n_rows < 0 || shard_vocab <= 0 || row_stride < shard_vocab || vocab_offset < 0) return PB_E_INVALID;
  if (cap < 1 || cap > PB_CAND_MAX_CAP) return PB_E_INVALID;
  if (vocab_offset + shard_vocab >= PB_MAX_VOCAB) return PB_E_TOO_LARGE;
  if (n_rows == 0) return PB_OK;
  if (!logits || !params || !out_records || !workspace) return PB_E_INVALID;
  if (n_rows > (int64_t)(0x7FFFFFFF / 8)) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(out_records) & 15) != 0) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return PB_E_INVALID;
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(logits) % es) != 0) return PB_E_INVALID;
  if (!groups_eligible(logits, row_stride, es, n_rows, shard_vocab) ||
      ws_bytes < group_plan(n_rows, shard_vocab, es).bytes)  // pb_candidates' launches
    return pb_candidates(logits, dtype, n_rows, shard_vocab, row_stride, row_index, params, vocab_offset, cap,
                         out_records, stream);
  Args a;
  a.logits = static_cast<const char*>(logits);
  a.n_rows = n_rows;
  a.vocab = shard_vocab;
  a.row_stride = row_stride;
  a.row_index = row_index;
  a.params = params;
  a.out_token = nullptr;
  a.out_info = nullptr;
  a.out_probs = nullptr;
  a.only_fallback = nullptr;
  a.complement = 0;
  a.cand_out = static_cast<uint8_t*>(out_records);
  a.cand_cap = cap;
  a.vocab_offset = vocab_offset;
  return run_groups_args(a, dtype, es, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
}

int pb_merge(const void* records, int32_t n_shards, int64_t n_rows, int32_t cap, const pb_row_params* params,
             int64_t* out_token, pb_row_info* out_info, void* stream) {
  if (n_shards < 1 || n_shards > 64 || n_rows < 0 || cap < 1 || cap > PB_CAND_MAX_CAP) return PB_E_INVALID;
  if (n_rows == 0) return PB_OK;
  if (!records || !params || !out_token) return PB_E_INVALID;
  if (n_rows > (int64_t)0x7FFFFFFF) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(records) & 15) != 0) return PB_E_INVALID;
  return launch_merge(static_cast<const uint8_t*>(records), n_shards, n_rows, cap, params, out_token, out_info,
                      static_cast<cudaStream_t>(stream));
}

int64_t pb_sample_ws_bytes(int64_t n_rows, int64_t vocab, int dtype) {
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es || n_rows < 0 || vocab <= 0) return PB_E_INVALID;
  // either launch: the balanced one (its grid never exceeds F_CPS CTAs per SM) or the two-pass one
  return std::max(ws_need(n_rows, (int64_t)F_CPS * sm_count()), group_plan(n_rows, vocab, es).bytes);
}

int pb_sample_ws(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                 const int32_t* row_index, const pb_row_params* params, int64_t* out_token, pb_row_info* out_info,
                 float* out_probs, void* workspace, int64_t ws_bytes, void* stream) {
  if (out_probs)  // probabilities come from the full-row path
    return pb_sample(logits, dtype, n_rows, vocab, row_stride, row_index, params, out_token, out_info, out_probs,
                     stream);
  if (n_rows < 0 || vocab <= 0 || row_stride < vocab) return PB_E_INVALID;
  if (vocab >= PB_MAX_VOCAB) return PB_E_TOO_LARGE;
  if (n_rows == 0) return PB_OK;
  if (!logits || !params || !out_token || !workspace) return PB_E_INVALID;
  if (n_rows > (int64_t)(0x7FFFFFFF / 8)) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return PB_E_INVALID;
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(logits) % es) != 0) return PB_E_INVALID;
  if (groups_eligible(logits, row_stride, es, n_rows, vocab) && ws_bytes >= group_plan(n_rows, vocab, es).bytes)
    return run_groups_dtype(logits, dtype, es, n_rows, vocab, row_stride, row_index, params, out_token, out_info,
                            static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
  const int64_t grid = balanced_grid(n_rows, vocab, es);
  if (ws_bytes < ws_need(n_rows, grid)) return PB_E_INVALID;
  return run_ws(logits, dtype, es, n_rows, vocab, row_stride, row_index, params, out_token, out_info,
                static_cast<uint8_t*>(workspace), grid, static_cast<cudaStream_t>(stream));
}

int64_t pb_sample_noalloc_max_bytes(void) { return NOALLOC_SCRATCH_BYTES; }

int pb_sample_noalloc(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                      const int32_t* row_index, const pb_row_params* params, int64_t* out_token,
                      pb_row_info* out_info, void* stream) {
  if (n_rows < 0 || vocab <= 0 || row_stride < vocab) return PB_E_INVALID;
  if (vocab >= PB_MAX_VOCAB) return PB_E_TOO_LARGE;
  if (n_rows == 0) return PB_OK;
  if (!logits || !params || !out_token) return PB_E_INVALID;
  if (n_rows > (int64_t)(0x7FFFFFFF / 8)) return PB_E_INVALID;
  const int es = (dtype == PB_DTYPE_F32) ? 4 : (dtype == PB_DTYPE_BF16 || dtype == PB_DTYPE_F16) ? 2 : 0;
  if (!es) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(logits) % es) != 0) return PB_E_INVALID;
  const bool groups = groups_eligible(logits, row_stride, es, n_rows, vocab) &&
                      group_plan(n_rows, vocab, es).bytes <= NOALLOC_SCRATCH_BYTES;
  const int64_t grid = balanced_grid(n_rows, vocab, es);
  if (!groups && ws_need(n_rows, grid) > NOALLOC_SCRATCH_BYTES) return PB_E_SCRATCH;
  uint8_t* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch);
  if (rc != PB_OK) return rc;
  if (groups)  // every group key pass 2 reads is written by pass 1 first
    return run_groups_dtype(logits, dtype, es, n_rows, vocab, row_stride, row_index, params, out_token, out_info,
                            scratch, static_cast<cudaStream_t>(stream));
  // the launches need no cleared memory: the arrival counters carry a check word (see f_arrive) and
  // every record is written before it is read
  return run_ws(logits, dtype, es, n_rows, vocab, row_stride, row_index, params, out_token, out_info, scratch,
                grid, static_cast<cudaStream_t>(stream));
}

uint32_t pb_key_of(float x) {
  if (x != x) return 0xFFFFFFFFu;
  uint32_t b;
  if (x == 0.0f) {
    b = 0;
  } else {
    memcpy(&b, &x, 4);
  }
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

int pb_stop_check(const int64_t* tokens, int64_t n_rows, const int32_t* row_state, const int32_t* stop_offsets,
                  const int32_t* stop_ids, int32_t eos_id, int32_t max_model_len, int8_t* out_reason, void* stream) {
  if (n_rows < 0) return PB_E_INVALID;
  if (n_rows == 0) return PB_OK;
  if (!tokens || !row_state || !stop_offsets || !out_reason) return PB_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(row_state) & 15) != 0) return PB_E_INVALID;
  if (n_rows > (int64_t)0x7FFFFFFF * 256) return PB_E_INVALID;
  stop_check_kernel<<<(unsigned)((n_rows + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      tokens, n_rows, reinterpret_cast<const int4*>(row_state), stop_offsets, stop_ids, eos_id, max_model_len,
      out_reason);
  return cudaGetLastError() == cudaSuccess ? PB_OK : PB_E_LAUNCH;
}

uint64_t pb_philox_u53(uint64_t seed, uint32_t step) { return philox_u53(seed, step); }

void pb_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) { philox4x32_10(ctr, key, out); }

float pb_exp(float d) {
  // host copy of exp_weight: same operation sequence
  if (!(d >= -87.0f)) return 0.0f;
  volatile float t = d * 0x1.715476p+0f;
  const float n = nearbyintf(t);
  float r = fmaf(-n, 0x1.62e43p-1f, d);
  r = fmaf(-n, -0x1.05c61p-29f, r);
  float p = 0x1.a01a02p-13f;
  p = fmaf(p, r, 0x1.6c16c2p-10f);
  p = fmaf(p, r, 0x1.111112p-7f);
  p = fmaf(p, r, 0x1.555556p-5f);
  p = fmaf(p, r, 0x1.555556p-3f);
  p = fmaf(p, r, 0x1.0p-1f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int32_t bits;
  memcpy(&bits, &p, 4);
  bits += ((int32_t)n) << 23;
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

const char* pb_strerror(int code) {
  switch (code) {
    case PB_OK: return "ok";
    case PB_E_INVALID: return "invalid argument";
    case PB_E_TOO_LARGE: return "vocabulary too large (must be < 2^24)";
    case PB_E_LAUNCH: return "kernel launch failed";
    case PB_E_DEVICE: return "device configuration failed";
    case PB_E_SCRATCH: return "batch needs more scratch than pb_sample_noalloc's fixed array holds";
    default: return "unknown error";
  }
}

int pb_version(void) { return 100; }

}  // extern "C"
