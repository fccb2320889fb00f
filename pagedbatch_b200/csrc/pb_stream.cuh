// Streaming kernel of the B200 sampler: persistent, one CTA per SM, warp-specialised.
//
// Included by pb_sample.cu inside its anonymous namespace (it shares the key, weight and
// selection helpers defined there). It settles the rows the engine samples most: greedy rows and
// top-k rows with 0 < top_k <= F_KMAX (with or without top-p), every one of them exactly as
// pb_sample's cluster kernel does (pagedbatch/sampling.py:12-27 in the fixed arithmetic stated in
// include/pagedbatch_b200.h). Other rows, and rows whose data it cannot settle (NaN or +inf values,
// more candidates than its buffers hold), it leaves to the cluster kernel, which runs next on the
// same stream and samples only those.
//
// CTA g takes rows g, g + grid, g + 2 grid, ... (whole rows). Warps:
//   * warp F_PROD (lane 0): the producer. Streams every chunk of the CTA's rows, one row after the
//     other, HBM -> a ring of F_NSTAGE 32 KB shared-memory stages with 1-D bulk copies (TMA engine,
//     no multicast), waiting on each stage's "empty" mbarrier and arming its "full" one with the
//     copy's byte count. It runs ahead across row boundaries, so the next row's first chunks are in
//     flight while a row is closed.
//   * warps 0..15: the consumers. Per chunk they wait on the stage's full barrier, copy their vectors
//     to registers, arrive on its empty barrier (nothing else), and track the row's max, its first
//     maximum (greedy rows) and the candidates >= a running threshold (top-k rows) in per-thread
//     slots; they meet (named barrier 1) only for the first threshold of a row and at checkpoints.
//     At the end of a top-k row they hand the candidates to a finisher through one of the list
//     buffers, then go straight on to the next row.
//   * warps F_FIN..: the finishers (rows alternate between them). For each handed-off row: the
//     exact k-th key, the survivors, their order (key desc, index asc), fixed-point weights, the
//     top-p cut and the inverse-CDF draw, all in one warp, while the consumers stream on.
// Every wait is bounded; a wait that gives up makes the whole CTA stop, let its issued copies land,
// and report PB_ROW_TIMEOUT for its rows.

constexpr int F_CW = 16;                    // consumer warps (barrier group 2: 512 threads)
constexpr int F_CT = F_CW * 32;             // consumer threads
constexpr int F_PROD = F_CW;                // producer warp
constexpr int F_NF = 2;                     // finisher warps (rows alternate between them)
constexpr int F_NB = 2 * F_NF;              // list buffers (two per finisher)
constexpr int F_FIN = F_CW + 1;             // first finisher warp
constexpr int F_THREADS = (F_CW + 1 + F_NF) * 32;
constexpr int F_CHUNK = CHUNK_BYTES;        // bytes per staged chunk (32 KB)
constexpr int F_NSTAGE = 4;                 // 128 KB of copies in flight per SM
constexpr int F_RING = F_NSTAGE * F_CHUNK;
constexpr int F_LCAP = 512;                 // candidates one row hands to the finisher
constexpr int F_KMAX = OFFER_PREFER;        // largest top_k settled here (thresholds from the offer bound)
constexpr int F_SMAX = 256;                 // survivors the finisher orders
constexpr int F_VSL = 8;                    // 16-byte vectors each consumer thread can hold as candidates
constexpr int F_CAND = F_VSL * F_CT * 16 + F_VSL * F_CT * 4;  // the vectors and their first element's index
constexpr int F_SMEM = F_RING + F_CAND + F_NB * F_LCAP * 8;
constexpr int64_t F_RETRY = -2;             // out_token mark: the cluster kernel samples this row
constexpr int32_t F_CAND_RETRY = 0x400;     // the same mark in a shard record's flags
static_assert(F_SMEM <= 227 * 1024, "one CTA per SM");
static_assert(F_SMAX <= F_LCAP && F_LCAP % 32 == 0, "finisher layout");

enum : int { F_NONE = 0, F_GREEDY = 1, F_FILTER = 2 };

// What the streaming kernel does with a row (the cluster kernel uses the same test to skip it):
// rejected parameters, temperature-only and top-p-only rows, top_k above F_KMAX and bad uniforms
// go to the cluster kernel.
__device__ __forceinline__ int fast_mode(const pb_row_params& p, int64_t V) {
  const bool bad = !(p.temperature >= 0.0) || !(p.top_p > 0.0 && p.top_p <= 1.0) || p.top_k < 0;
  if (bad) return F_NONE;
  if (p.temperature == 0.0) return F_GREEDY;
  if (p.top_k > 0 && p.top_k <= F_KMAX && (int64_t)p.top_k < V && p.uniform >= 0.0 && p.uniform < 1.0)
    return F_FILTER;
  return F_NONE;
}

// Wait for the programmatic launch dependency (a no-op for a kernel launched without one).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

struct FastArgs {
  const char* logits;
  int64_t n_rows, vocab, row_stride;
  const int32_t* row_index;
  const pb_row_params* params;
  int64_t* out_token;
  pb_row_info* out_info;
  uint8_t* cand_out;  // vocabulary-parallel shard mode (else null)
  int32_t cand_cap;
  int64_t vocab_offset;
  int32_t poll_limit;  // polls of the consumers' waits on staged chunks (WAIT_POLLS; 0 makes them give up)
};

// One row handed from the consumers to the finisher.
struct FastList {
  int64_t item;
  int32_t n;      // candidates in the list
  int32_t retry;  // the cluster kernel samples this row
  float m;        // largest scaled key
  int32_t pad;
};

struct FastShared {
  uint64_t full[F_NSTAGE], empty[F_NSTAGE];  // ring: copy landed / every consumer warp done with it
  uint64_t lfull[F_NB], lfree[F_NB];         // list buffers: handed off / finisher done with it
  int64_t issued[F_NSTAGE];                  // last chunk issued into each stage (-1: none)
  volatile int32_t abort;                    // a wait gave up: every role stops
  FastList lh[F_NB];
  float wbest[F_CW], wmx[F_CW];
  uint32_t wbidx[F_CW];
  uint32_t cpb[2][F_CW];  // per checkpoint (alternating): each consumer warp's share of the offer bound
  uint32_t ob[F_CW];      // each consumer warp's share of a row's first threshold
  uint32_t s32[F_CW + 2]; // scan scratch of the consumer group
  int32_t cp_flags[3];    // checkpoint flags (timeout 4, overflow 2), rotating so a reset never races a write
  int32_t lfail;          // the wait for a free list buffer gave up (written before a barrier)
};

// Bounded wait that also gives up once another role has set `abort`.
__device__ __forceinline__ bool f_wait(uint64_t* bar, uint32_t parity, int limit, volatile int32_t* abort) {
  for (int i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
  }
  return false;
}

// A whole row: scalar head up to the first 16-byte boundary, 16-byte vectors, scalar tail.
template <typename T>
struct FRow {
  const T* row;
  int64_t head_n, vec_e0, nvec, tail_e0, tail_n;
};

template <typename T>
__device__ __forceinline__ FRow<T> f_row(const FastArgs& a, int64_t item) {
  constexpr int ES = Elem<T>::ES, EPV = Elem<T>::EPV;
  FRow<T> r;
  const int64_t rid = a.row_index ? (int64_t)a.row_index[item] : item;
  r.row = reinterpret_cast<const T*>(a.logits) + rid * a.row_stride;
  const int64_t V = a.vocab;
  int64_t head = (int64_t)(((16 - (reinterpret_cast<uintptr_t>(r.row) & 15)) & 15) / ES);
  if (head > V) head = V;
  r.head_n = head;
  r.vec_e0 = head;
  r.nvec = (V - head) / EPV;
  r.tail_e0 = head + r.nvec * EPV;
  r.tail_n = V - r.tail_e0;
  return r;
}

__device__ __forceinline__ void f_mark_retry(const FastArgs& a, int64_t item) {
  if (a.cand_out)
    reinterpret_cast<pb_cand_header*>(a.cand_out + item * record_bytes(a.cand_cap))->flags = F_CAND_RETRY;
  else
    a.out_token[item] = F_RETRY;
}

// ---- producer ------------------------------------------------------------------------------------

template <typename T>
__device__ void f_producer(const FastArgs& a, FastShared& fs, uint4* ring) {
  constexpr int CV = F_CHUNK / 16;
  const uint64_t pol = l2_policy_evict_first();
  uint32_t seq = 0;
  for (int64_t item = blockIdx.x; item < a.n_rows; item += gridDim.x) {
    if (fast_mode(a.params[item], a.vocab) == F_NONE) continue;
    const FRow<T> r = f_row<T>(a, item);
    const int nvec = (int)r.nvec;
    const uint4* src = reinterpret_cast<const uint4*>(r.row + r.vec_e0);
    for (int c = 0; c * CV < nvec; ++c, ++seq) {
      const int st = (int)(seq % F_NSTAGE);
      // a fresh barrier counts as having completed the phase before its first one
      if (!f_wait(&fs.empty[st], ((seq / F_NSTAGE) & 1) ^ 1, WAIT_POLLS, &fs.abort)) {
        fs.abort = 1;
        return;
      }
      const int nv = min(CV, nvec - c * CV);
      fs.issued[st] = seq;
      fence_proxy_async();
      mbar_expect_tx(&fs.full[st], (uint32_t)(nv * 16));
      bulk_load(ring + st * CV, src + (int64_t)c * CV, (uint32_t)(nv * 16), &fs.full[st], pol);
    }
  }
}

// ---- finisher -----------------------------------------------------------------------------------

// One register value of a[] chosen by a runtime index (unrolled select: no local memory).
template <int NPL>
__device__ __forceinline__ uint64_t reg_at(const uint64_t (&a)[NPL], int r) {
  uint64_t v = 0;
#pragma unroll
  for (int i = 0; i < NPL; ++i)
    if (i == r) v = a[i];
  return v;
}

// Sort 32 * NPL composites descending in one warp's registers: lane l holds positions
// l * NPL .. l * NPL + NPL - 1 (a bitonic network; 0 sorts last). All 32 lanes call.
template <int NPL>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&a)[NPL]) {
  constexpr int N = 32 * NPL;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= NPL) {
#pragma unroll
        for (int r = 0; r < NPL; ++r) {
          const int pos = lane * NPL + r;
          const bool desc = (pos & k) == 0, lower = (pos & j) == 0;
          const uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, a[r], j / NPL);
          a[r] = (lower == desc) ? max(a[r], o) : min(a[r], o);
        }
      } else {
#pragma unroll
        for (int r = 0; r < NPL; ++r) {
          if ((r & j) == 0) {
            const bool desc = ((lane * NPL + r) & k) == 0;
            const uint64_t x = a[r], y = a[r | j];
            if (desc ? (x < y) : (x > y)) {
              a[r] = y;
              a[r | j] = x;
            }
          }
        }
      }
    }
  }
}

// The composite at sorted position `pos` (every lane gets it).
template <int NPL>
__device__ __forceinline__ uint64_t warp_at(const uint64_t (&a)[NPL], int pos) {
  return __shfl_sync(0xFFFFFFFFu, reg_at(a, pos % NPL), pos / NPL);
}

// Over the first n sorted composites (scaled key desc, index asc) in registers: fixed-point
// weights, inclusive scan, the top-p cut and the draw. Same decisions as warp_finish and
// finish_survivors. Lane 0 receives the result in *f. All 32 lanes call.
template <int NPL>
__device__ void warp_finish_sorted(const uint64_t (&a)[NPL], int n, float m, bool topp, float pf, uint64_t u53,
                                   Finish* f) {
  const int lane = threadIdx.x & 31;
  uint64_t q[NPL];
  uint64_t s = 0;
#pragma unroll
  for (int r = 0; r < NPL; ++r) {
    q[r] = (lane * NPL + r < n) ? weight_q(value_of(comp_key(a[r])), m) : 0ull;
    s += q[r];
  }
  const uint64_t incl = warp_incl_scan(s);
  const uint64_t excl = incl - s;
  const uint64_t zq = __shfl_sync(0xFFFFFFFFu, incl, 31);
  // first position whose inclusive prefix exceeds t (t < total), and that prefix
  auto find = [&](uint64_t t, uint64_t* at) -> int {
    const bool here = excl <= t && t < incl;
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, here);
    if (bal == 0) return -1;
    int pos = -1;
    uint64_t inc = 0, run = excl;
#pragma unroll
    for (int r = 0; r < NPL; ++r) {
      run += q[r];
      if (pos < 0 && run > t) {
        pos = lane * NPL + r;
        inc = run;
      }
    }
    const int src = __ffs(bal) - 1;
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
  const uint32_t tk = comp_key(warp_at(a, last));
  const uint64_t tok = warp_at(a, pick);
  int c = 0;
#pragma unroll
  for (int r = 0; r < NPL; ++r) c += (lane * NPL + r <= last && comp_key(a[r]) == tk) ? 1 : 0;
  const int n_tie = warp_sum(c);
  if (lane == 0) {
    f->ok = ok;
    f->last = last;
    f->n_tie = n_tie;
    f->token = ok ? (int64_t)comp_idx(tok) : -1;
    f->thr_key = tk;
    f->zq = zq;
    f->kept = kept;
  }
}

// Settle a top-k row from n <= 32 * NPL candidates at L (composites of raw key and index, or of
// the scaled key with SCALED, which hold every survivor): scaled keys, one sort, the kq-th scaled key at position kq - 1 (x / T is
// monotone), the survivors (the prefix with key >= it, ties included), then the record (shard
// mode) or the draw. All 32 lanes call.
template <int NPL, bool SCALED = false>
__device__ void finish_list(const FastArgs& a, const pb_row_params& p, int64_t item, const uint64_t* L, int n,
                            float m, int32_t flags = PB_PATH_SMALL | PB_PATH_STREAM) {
  const int lane = threadIdx.x & 31;
  const float tf = (float)p.temperature;
  uint64_t v[NPL];
#pragma unroll
  for (int r = 0; r < NPL; ++r) {
    const int pos = lane * NPL + r;
    uint64_t c = 0;
    if (pos < n) {
      const uint64_t raw = L[pos];
      c = SCALED ? raw : compose(key_of(__fdiv_rn(value_of(comp_key(raw)), tf)), comp_idx(raw));
    }
    v[r] = c;
  }
  warp_sort_desc<NPL>(v);
  const int kq = min(p.top_k, n);
  const uint32_t kth_s = comp_key(warp_at(v, kq - 1));
  int cnt = 0;
#pragma unroll
  for (int r = 0; r < NPL; ++r) cnt += (lane * NPL + r < n && comp_key(v[r]) >= kth_s) ? 1 : 0;
  const int S = warp_sum(cnt);  // survivors: the sorted prefix [0, S)
  if (a.cand_out) {
    // vocabulary-parallel shard: publish the survivors (global indices), as the cluster kernel does
    uint8_t* rec = a.cand_out + item * record_bytes(a.cand_cap);
    uint64_t* ent = reinterpret_cast<uint64_t*>(rec + sizeof(pb_cand_header));
    const bool fits = S <= min(a.cand_cap, KCAP);
    if (fits) {
#pragma unroll
      for (int r = 0; r < NPL; ++r) {
        const int pos = lane * NPL + r;
        if (pos < S) ent[pos] = compose(comp_key(v[r]), comp_idx(v[r]) + (uint32_t)a.vocab_offset);
      }
    }
    if (lane == 0) {
      pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(rec);
      hd->count = fits ? S : 0;
      hd->flags = fits ? 0 : PB_CAND_FALLBACK;
      hd->max_key = m;
      hd->reserved = 0;
    }
    return;
  }
  const bool topp = p.top_p < 1.0 && (float)p.top_p < 1.0f;
  Finish f;
  warp_finish_sorted<NPL>(v, S, m, topp, (float)p.top_p, (uint64_t)(p.uniform * 0x1p53), &f);
  if (lane == 0) {
    a.out_token[item] = f.ok ? f.token : -1;
    if (a.out_info) {
      pb_row_info* o = a.out_info + item;
      o->thr_key = f.thr_key;
      o->n_tie_kept = f.n_tie;
      o->kept_count = f.last + 1;
      o->status = f.ok ? PB_ROW_OK : PB_ROW_INTERNAL;
      o->max_key = m;
      o->flags = flags;
      o->z_q = f.zq;
      o->kept_q = f.kept;
    }
  }
}

// Settle one handed-off top-k row in the finisher warp. L holds h.n composites (raw key, index).
// Up to F_SMAX candidates go straight to one sort; a longer list is first cut to its survivors by
// a bisection for the exact k-th raw key.
__device__ void f_finish_row(const FastArgs& a, const pb_row_params& p, const FastList& h, uint64_t* L) {
  const int lane = threadIdx.x & 31;
  const int64_t item = h.item;
  if (h.retry) {
    if (lane == 0) f_mark_retry(a, item);
    return;
  }
  int n = h.n;
  if (n > F_SMAX) {
    constexpr int NPL = F_LCAP / 32;
    const float tf = (float)p.temperature;
    uint64_t c[NPL];
    uint32_t kk[NPL];
    uint32_t mn = 0xFFFFFFFFu, mx = 0;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int i = j * 32 + lane;
      c[j] = (i < n) ? L[i] : 0ull;
      kk[j] = comp_key(c[j]);  // 0 (below every key) for padding
      if (i < n) mn = min(mn, kk[j]);
      mx = max(mx, kk[j]);
    }
    mn = __reduce_min_sync(0xFFFFFFFFu, mn);
    mx = __reduce_max_sync(0xFFFFFFFFu, mx);
    // exact kq-th largest raw key: the largest X with #(keys >= X) >= kq (always a key of the list)
    const uint32_t kq = (uint32_t)min(p.top_k, n);
    uint32_t lo = mn;
    uint64_t hi = (uint64_t)mx + 1;
    while (hi - lo > 1) {
      const uint32_t mid = (uint32_t)(lo + ((hi - lo) >> 1));
      uint32_t cnt = 0;
#pragma unroll
      for (int j = 0; j < NPL; ++j) cnt += (kk[j] >= mid) ? 1u : 0u;
      cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
      if (cnt >= kq) lo = mid;
      else hi = mid;
    }
    // survivors keep their raw composites: scaled key >= the scaled k-th key
    const uint32_t kth_s = key_of(__fdiv_rn(value_of(lo), tf));
    bool sv[NPL];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      sv[j] = j * 32 + lane < n && (kk[j] >= lo || key_of(__fdiv_rn(value_of(kk[j]), tf)) >= kth_s);
      cnt += sv[j] ? 1 : 0;
    }
    const int incl = warp_incl_scan(cnt);
    n = __shfl_sync(0xFFFFFFFFu, incl, 31);
    __syncwarp();  // every lane holds its list entries in registers: L may be overwritten
    int w = incl - cnt;
#pragma unroll
    for (int j = 0; j < NPL; ++j)
      if (sv[j]) L[w++] = c[j];
    __syncwarp();
    if (n > F_SMAX) {
      if (lane == 0) f_mark_retry(a, item);
      return;
    }
  }
  if (n <= 64) finish_list<2>(a, p, item, L, n, h.m);
  else if (n <= 128) finish_list<4>(a, p, item, L, n, h.m);
  else finish_list<8>(a, p, item, L, n, h.m);
}

template <typename T>
__device__ void f_finisher(const FastArgs& a, FastShared& fs, uint64_t* lists, int fin) {
  const int lane = threadIdx.x & 31;
  uint32_t lseq = 0;  // top-k rows of this CTA so far (this warp takes every F_NF-th)
  for (int64_t item = blockIdx.x; item < a.n_rows; item += gridDim.x) {
    const pb_row_params p = a.params[item];
    if (fast_mode(p, a.vocab) != F_FILTER) continue;
    const uint32_t mine = lseq++;
    if ((int)(mine % F_NF) != fin) continue;
    const int b = (int)(mine % F_NB);
    if (!__all_sync(0xFFFFFFFFu, f_wait(&fs.lfull[b], (mine / F_NB) & 1, WAIT_POLLS, &fs.abort))) {
      if (lane == 0) fs.abort = 1;
      return;
    }
    const FastList h = fs.lh[b];
    f_finish_row(a, p, h, lists + b * F_LCAP);
    __syncwarp();  // the list is read and rewritten before the consumers may refill it
    if (lane == 0) mbar_arrive(&fs.lfree[b]);
  }
}

// ---- consumers ------------------------------------------------------------------------------------

// The offer bound of the consumer group: every thread offers one key (0: none); each warp sorts
// its 32 offers (bitonic, in registers) and publishes its ceil(k / F_CW)-th largest; the smallest
// over the warps is reached by at least k offers. Every thread returns the same key. One barrier;
// `slot` must not be read by another call until a later barrier.
__device__ __forceinline__ uint32_t f_offer_bound(uint32_t key, int k, uint32_t* slot, FastShared& fs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, key, stride);
      const bool desc = (lane & size) == 0, lower = (lane & stride) == 0;
      key = (lower == desc) ? max(key, o) : min(key, o);
    }
  }
  const uint32_t kj = __shfl_sync(0xFFFFFFFFu, key, (k + F_CW - 1) / F_CW - 1);
  if (lane == 0) slot[warp] = kj;
  bsync<2>();
  uint32_t mn = 0xFFFFFFFFu;
#pragma unroll
  for (int w = 0; w < F_CW; ++w) mn = min(mn, slot[w]);
  return mn;
}


// Candidates of a top-k row are whole 16-byte vectors: a thread keeps (in shared memory) every
// vector of its own that holds a value at or above the threshold, with the index of its first
// element. Storing a vector costs no per-element work in the streaming loop; the values are
// looked at one by one only when the threshold rises and when the row is handed off.

// Checkpoints of a row (after chunk c): after 4 chunks (the first threshold, from one chunk, is
// loose), then every 12 chunks (384 KB), and after the last chunk.
__device__ __forceinline__ bool f_checkpoint(int c, int nch) {
  const int n = c + 1;
  return n == nch || (n % 12) == 4;
}

// Largest element of a vector (NaN-propagating), as fp32.
template <typename T>
__device__ __forceinline__ float vec_max(uint4 v) {
  using E = Elem<T>;
  return E::word_max(E::max2(E::max2(v.x, v.y), E::max2(v.z, v.w)));
}

// w[j] for a runtime j (an unrolled select: the array stays in registers)
template <int N>
__device__ __forceinline__ uint4 reg_pick(const uint4 (&w)[N], int j) {
  uint4 v = w[0];
#pragma unroll
  for (int i = 1; i < N; ++i)
    if (i == j) v = w[i];
  return v;
}

template <typename T>
__device__ void f_consumers(const FastArgs& a, FastShared& fs, const uint4* ring, uint4* cand,
                            uint64_t* lists) {
  using E = Elem<T>;
  constexpr int EPV = E::EPV;
  constexpr int CV = F_CHUNK / 16;  // vectors per chunk
  constexpr int VPT = CV / F_CT;          // vectors per thread per chunk
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t V = a.vocab;
  uint4* vs = cand;                                                // held vectors: slot j of thread t at j * F_CT + t
  uint32_t* vb = reinterpret_cast<uint32_t*>(cand + F_VSL * F_CT);  // index of each held vector's first element
  uint32_t seq = 0, lseq = 0;
  int cp = 0;              // checkpoints passed (their flag words rotate over three slots)
  bool timed_out = false;  // this warp gave up waiting on a staged chunk (warp-uniform)
  bool stop = false;       // the CTA gave up (uniform over the consumers)
  if (tid == 0)
    for (int i = 0; i < 3; ++i) fs.cp_flags[i] = 0;
  bsync<2>();
  for (int64_t item = blockIdx.x; item < a.n_rows && !stop; item += gridDim.x) {
    const pb_row_params p = a.params[item];
    const int mode = fast_mode(p, V);
    if (mode == F_NONE) continue;
    const bool greedy = mode == F_GREEDY;
    const float tf = (float)p.temperature;
    const int k = p.top_k;
    const FRow<T> r = f_row<T>(a, item);
    const int nvec = (int)r.nvec;
    const int nch = (nvec + CV - 1) / CV;
    float runmax = -INFINITY, bestv = -INFINITY;
    uint32_t bidx = 0xFFFFFFFFu;
    int nc = 0;             // vectors this thread holds
    bool ovf = false;       // a vector of this thread found no free slot
    bool row_ovf = false;   // some thread overflowed (uniform)
    float t = -INFINITY;    // candidate threshold (a tie floor); changes only at barriers
    const uint32_t e_base = (uint32_t)r.vec_e0 + (uint32_t)tid * EPV;  // element of vector tid of chunk 0
    for (int c = 0; c < nch; ++c, ++seq) {
      const int st = (int)(seq % F_NSTAGE);
      if (!timed_out)
        timed_out = !__all_sync(0xFFFFFFFFu, f_wait(&fs.full[st], (seq / F_NSTAGE) & 1, a.poll_limit, &fs.abort));
      const int nv = min(CV, nvec - c * CV);
      const uint4* buf = ring + st * CV;
      // this thread's vectors of the chunk as raw words (-inf past the chunk's end)
      uint4 w[VPT];
      if (nv == CV && !timed_out) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) w[j] = buf[j * F_CT + tid];
      } else {
        const uint4 pad = make_uint4(E::NEG_INF_WORD, E::NEG_INF_WORD, E::NEG_INF_WORD, E::NEG_INF_WORD);
#pragma unroll
        for (int j = 0; j < VPT; ++j) w[j] = (j * F_CT + tid < nv && !timed_out) ? buf[j * F_CT + tid] : pad;
      }
      __syncwarp();
      if (lane == 0 && !timed_out) mbar_arrive(&fs.empty[st]);  // the vectors are in registers
      // per-vector and per-chunk maxima on the packed words (NaN-propagating)
      uint32_t vm2[VPT];
#pragma unroll
      for (int j = 0; j < VPT; ++j) vm2[j] = E::max2(E::max2(w[j].x, w[j].y), E::max2(w[j].z, w[j].w));
      uint32_t t2 = vm2[0];
#pragma unroll
      for (int j = 1; j < VPT; ++j) t2 = E::max2(t2, vm2[j]);
      const float tm = E::word_max(t2);
      runmax = fmax_nan(runmax, tm);
      if (greedy) {
        if (tm > bestv) {  // a new maximum: its first position among this thread's elements
          uint32_t hit = 0;
#pragma unroll
          for (int j = 0; j < VPT; ++j) hit |= (E::word_max(vm2[j]) == tm) ? (1u << j) : 0u;
          const int j = __ffs(hit) - 1;
          float x[EPV];
          E::unpack(reg_pick(w, j), x);
          int jj = EPV - 1;
#pragma unroll
          for (int q = EPV - 1; q >= 0; --q)
            if (x[q] == tm) jj = q;
          bidx = e_base + (uint32_t)((c * CV + j * F_CT) * EPV + jj);
          bestv = tm;
        }
      } else {
        if (c == 0) {
          // first threshold: a lower bound of the row's k-th value from this chunk (each warp's
          // ceil(k/8)-th largest per-thread maximum, the smallest over the warps), as a tie floor
          uint32_t lo = 0;
          if (nv * EPV >= k) lo = f_offer_bound(key_of(tm), k, fs.ob, fs);  // nv is the same for all
          t = (lo > KEY_NEG_INF) ? tie_floor(value_of(lo), tf) : -INFINITY;  // (same in every thread)
        }
        if (!row_ovf && !timed_out && tm >= t) {
          // keep every vector that reaches t: predicated stores into the next free slots
          uint32_t hit = 0;  // (padding holds -inf: only real vectors)
#pragma unroll
          for (int j = 0; j < VPT; ++j) hit |= (E::word_max(vm2[j]) >= t && j * F_CT + tid < nv) ? (1u << j) : 0u;
          while (hit) {  // usually one vector
            const int j = __ffs(hit) - 1;
            hit &= hit - 1;
            const int sl = min(nc, F_VSL - 1);  // (a store past the last slot only happens on overflow)
            vs[sl * F_CT + tid] = reg_pick(w, j);
            vb[sl * F_CT + tid] = e_base + (uint32_t)((c * CV + j * F_CT) * EPV);
            ++nc;
          }
          if (nc > F_VSL) {
            ovf = true;
            nc = F_VSL;
          }
        }
      }
      if (!greedy && f_checkpoint(c, nch)) {
        // checkpoint (one barrier): agree on timeouts and overflow, and raise the threshold by the
        // offer bound of the values held (every thread offers its largest; each warp's
        // ceil(k/8)-th largest offer, the smallest over the warps, is reached by at least k of
        // them), then each thread drops its vectors below the new threshold
        float top = -INFINITY;
        for (int j = 0; j < nc; ++j) top = fmax_nan(top, vec_max<T>(vs[j * F_CT + tid]));
        uint32_t key = nc > 0 ? key_of(top) : 0u;
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
          for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, key, stride);
            const bool desc = (lane & size) == 0, lower = (lane & stride) == 0;
            key = (lower == desc) ? max(key, o) : min(key, o);
          }
        }
        const uint32_t kj = __shfl_sync(0xFFFFFFFFu, key, (k + F_CW - 1) / F_CW - 1);
        const bool wovf = __any_sync(0xFFFFFFFFu, ovf);
        if (lane == 0) {
          fs.cpb[cp & 1][warp] = kj;
          const int mine = ((timed_out || fs.abort) ? 4 : 0) | (wovf ? 2 : 0);
          if (mine) atomicOr(&fs.cp_flags[cp % 3], mine);
        }
        bsync<2>();
        const int f = fs.cp_flags[cp % 3];
        uint32_t lo = 0xFFFFFFFFu;
#pragma unroll
        for (int w2 = 0; w2 < F_CW; ++w2) lo = min(lo, fs.cpb[cp & 1][w2]);
        if (tid == 0) fs.cp_flags[(cp + 2) % 3] = 0;
        ++cp;
        if (f & 4) {
          stop = true;
          break;
        }
        if (f & 2) row_ovf = true;
        if (!row_ovf && lo > KEY_NEG_INF && lo != 0xFFFFFFFFu) {
          t = fmaxf(t, tie_floor(value_of(lo), tf));  // (same in every thread)
          int kept = 0;
          for (int j = 0; j < nc; ++j) {
            const uint4 v = vs[j * F_CT + tid];
            if (vec_max<T>(v) >= t) {
              if (kept != j) {
                vs[kept * F_CT + tid] = v;
                vb[kept * F_CT + tid] = vb[j * F_CT + tid];
              }
              ++kept;
            }
          }
          nc = kept;
        }
      }
    }
    if (stop) break;
    // scalar head and tail: greedy rows compare them (first index wins among equal values); top-k
    // rows collect them below, as single elements
    for (int64_t e = tid; e < r.head_n + r.tail_n; e += F_CT) {
      const int64_t ei = (e < r.head_n) ? e : r.tail_e0 + (e - r.head_n);
      const float xv = E::ld(r.row + ei);
      runmax = fmax_nan(runmax, xv);
      if (greedy && (xv > bestv || (xv == bestv && (uint32_t)ei < bidx))) {
        bestv = xv;
        bidx = (uint32_t)ei;
      }
    }

    if (greedy) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xFFFFFFFFu, bestv, o);
        const uint32_t i2 = __shfl_xor_sync(0xFFFFFFFFu, bidx, o);
        if (v2 > bestv || (v2 == bestv && i2 < bidx)) {
          bestv = v2;
          bidx = i2;
        }
        runmax = fmax_nan(runmax, __shfl_xor_sync(0xFFFFFFFFu, runmax, o));
      }
      if (lane == 0) {
        fs.wbest[warp] = bestv;
        fs.wbidx[warp] = bidx;
        fs.wmx[warp] = runmax;
        if (timed_out || fs.abort) atomicOr(&fs.cp_flags[cp % 3], 4);
      }
      bsync<2>();
      {
        const int f = fs.cp_flags[cp % 3];
        if (tid == 0) fs.cp_flags[(cp + 2) % 3] = 0;
        ++cp;
        if (f & 4) {
          stop = true;
          break;
        }
      }
      if (tid == 0) {
        for (int w = 1; w < F_CW; ++w) {
          if (fs.wbest[w] > bestv || (fs.wbest[w] == bestv && fs.wbidx[w] < bidx)) {
            bestv = fs.wbest[w];
            bidx = fs.wbidx[w];
          }
          runmax = fmax_nan(runmax, fs.wmx[w]);
        }
        if (runmax != runmax) {
          f_mark_retry(a, item);  // a NaN: the cluster kernel finds the first one
        } else {
          const uint32_t tok = (bidx == 0xFFFFFFFFu) ? 0u : bidx;  // every value -inf: the first index
          if (a.cand_out) {
            uint8_t* rec = a.cand_out + item * record_bytes(a.cand_cap);
            reinterpret_cast<uint64_t*>(rec + sizeof(pb_cand_header))[0] =
                compose(key_of(bestv), tok + (uint32_t)a.vocab_offset);
            pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(rec);
            hd->count = 1;
            hd->flags = PB_CAND_GREEDY;
            hd->max_key = bestv;
            hd->reserved = 0;
          } else {
            a.out_token[item] = tok;
            if (a.out_info) {
              pb_row_info* o = a.out_info + item;
              o->thr_key = key_of(bestv);
              o->n_tie_kept = 1;
              o->kept_count = 1;
              o->status = PB_ROW_OK;
              o->max_key = bestv;
              o->flags = PB_PATH_GREEDY | PB_PATH_STREAM;
              o->z_q = 0;
              o->kept_q = 0;
            }
          }
        }
      }
      bsync<2>();  // fs.wbest / wbidx / wmx are read before the next row writes them
      continue;
    }

    // top-k row: the values >= t of the held vectors (the last checkpoint raised t after the last
    // chunk) and of the scalar head and tail go to the finisher
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) runmax = fmax_nan(runmax, __shfl_xor_sync(0xFFFFFFFFu, runmax, o));
    if (lane == 0) fs.wmx[warp] = runmax;
    uint32_t cnt = 0;
    if (!row_ovf) {
      for (int j = 0; j < nc; ++j) {
        float x[EPV];
        E::unpack(vs[j * F_CT + tid], x);
#pragma unroll
        for (int q = 0; q < EPV; ++q) cnt += (x[q] >= t) ? 1u : 0u;
      }
      for (int64_t e = tid; e < r.head_n + r.tail_n; e += F_CT) {
        const int64_t ei = (e < r.head_n) ? e : r.tail_e0 + (e - r.head_n);
        cnt += (E::ld(r.row + ei) >= t) ? 1u : 0u;
      }
    }
    const int b = (int)(lseq % F_NB);
    if (tid == 0) fs.lfail = f_wait(&fs.lfree[b], ((lseq / F_NB) & 1) ^ 1, WAIT_POLLS, &fs.abort) ? 0 : 1;
    uint32_t total;
    uint32_t pos = block_excl_scan<uint32_t, F_CT, 2>(cnt, fs.s32, &total);  // (publishes fs.wmx, lfail)
    if (fs.lfail) {
      stop = true;
      if (tid == 0) fs.abort = 1;
      break;
    }
    float mraw = fs.wmx[0];
#pragma unroll
    for (int w = 1; w < F_CW; ++w) mraw = fmax_nan(mraw, fs.wmx[w]);
    const float m = __fdiv_rn(mraw, tf);
    const uint32_t mk = key_of(m);
    const bool retry = row_ovf || total == 0 || total > (uint32_t)F_LCAP || mk >= KEY_POS_INF || mk <= KEY_NEG_INF;
    if (!retry) {
      uint64_t* L = lists + b * F_LCAP;
      for (int j = 0; j < nc; ++j) {
        float x[EPV];
        E::unpack(vs[j * F_CT + tid], x);
        const uint32_t e0 = vb[j * F_CT + tid];
#pragma unroll
        for (int q = 0; q < EPV; ++q)
          if (x[q] >= t) L[pos++] = compose(key_of(x[q]), e0 + (uint32_t)q);
      }
      for (int64_t e = tid; e < r.head_n + r.tail_n; e += F_CT) {
        const int64_t ei = (e < r.head_n) ? e : r.tail_e0 + (e - r.head_n);
        const float xv = E::ld(r.row + ei);
        if (xv >= t) L[pos++] = compose(key_of(xv), (uint32_t)ei);
      }
    }
    bsync<2>();  // the list is written; every thread is done with fs.wmx and its vectors
    if (tid == 0) {
      FastList h;
      h.item = item;
      h.n = (int32_t)total;
      h.retry = retry ? 1 : 0;
      h.m = m;
      h.pad = 0;
      fs.lh[b] = h;
      __threadfence_block();
      mbar_arrive(&fs.lfull[b]);
    }
    ++lseq;
  }
  if (stop && tid == 0) fs.abort = 1;
}

// ---- the kernel ------------------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(F_THREADS, 1) stream_kernel(FastArgs a) {
  extern __shared__ __align__(128) unsigned char dyn[];
  __shared__ FastShared fs;
  uint4* ring = reinterpret_cast<uint4*>(dyn);
  uint4* cand = reinterpret_cast<uint4*>(dyn + F_RING);
  uint64_t* lists = reinterpret_cast<uint64_t*>(dyn + F_RING + F_CAND);
  const int tid = threadIdx.x, warp = tid >> 5;
  griddep_launch_dependents();  // the cluster kernel that follows may launch; it waits for this grid
  if (tid == 0) {
    for (int s = 0; s < F_NSTAGE; ++s) {
      mbar_init(&fs.full[s], 1);
      mbar_init(&fs.empty[s], F_CW);
      fs.issued[s] = -1;
    }
    for (int b = 0; b < F_NB; ++b) {
      mbar_init(&fs.lfull[b], 1);
      mbar_init(&fs.lfree[b], 1);
    }
    fs.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == F_PROD) {
    if ((tid & 31) == 0) f_producer<T>(a, fs, ring);
  } else if (warp >= F_FIN) {
    f_finisher<T>(a, fs, lists, warp - F_FIN);
  } else {
    f_consumers<T>(a, fs, ring, cand, lists);
  }
  __syncthreads();
  if (fs.abort && tid == 0) {
    // let every issued copy land before the shared memory is released, then report the CTA's rows
    for (int s = 0; s < F_NSTAGE; ++s)
      if (fs.issued[s] >= 0) mbar_wait_bounded(&fs.full[s], (uint32_t)((fs.issued[s] / F_NSTAGE) & 1), WAIT_POLLS);
    for (int64_t item = blockIdx.x; item < a.n_rows; item += gridDim.x) {
      if (fast_mode(a.params[item], a.vocab) == F_NONE) continue;
      if (a.cand_out) {
        pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(a.cand_out + item * record_bytes(a.cand_cap));
        hd->count = 0;
        hd->flags = PB_ROW_TIMEOUT;
        hd->max_key = 0.0f;
        hd->reserved = 0;
      } else {
        a.out_token[item] = -1;
        if (a.out_info) {
          pb_row_info* o = a.out_info + item;
          o->thr_key = 0;
          o->n_tie_kept = 0;
          o->kept_count = 0;
          o->status = PB_ROW_TIMEOUT;
          o->max_key = 0.0f;
          o->flags = PB_PATH_STREAM;
          o->z_q = 0;
          o->kept_q = 0;
        }
      }
    }
  }
}
