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
// Work is cut into segments (see "segments" below): whole rows, or, in the balanced mode of the
// workspace path, equal shares of the batch per CTA, so a row may be split into pieces over
// neighbouring CTAs. Warps:
//   * warp F_PROD (lane 0): the producer. Streams every chunk of the CTA's segments, one after the
//     other, HBM -> a ring of F_NSTAGE 32 KB shared-memory stages with 1-D bulk copies (TMA engine,
//     no multicast), waiting on each stage's "empty" mbarrier and arming its "full" one with the
//     copy's byte count. It runs ahead across segment boundaries.
//   * warps 0..15: the consumers. Per chunk they wait on the stage's full barrier, copy their vectors
//     to registers, arrive on its empty barrier (nothing else), and track the segment's max, its
//     first maximum (greedy rows) and the candidates >= a running threshold (top-k rows) in
//     per-thread slots; they meet (a bounded mbarrier barrier) only for the first threshold of a
//     top-k segment and at checkpoints. At the end of a segment each warp adds its part to one of
//     the list buffers on its own (shared-memory atomics reserve its place) and arrives on the
//     buffer's "full" barrier; no warp waits for another.
//   * warps F_FIN..: the finishers (segments alternate between them). For each segment: greedy rows
//     take the largest composite; top-k rows the exact k-th key, the survivors, their order (key
//     desc, index asc), fixed-point weights, the top-p cut and the inverse-CDF draw, all in one
//     warp, while the consumers stream on. A piece of a split row is published as a record and the
//     piece that arrives last merges the row.
// Every wait is bounded; a wait that gives up makes the whole CTA stop, let its issued copies land,
// and report PB_ROW_TIMEOUT for its rows.

#ifndef PB_STREAM_CTAS_PER_SM
#define PB_STREAM_CTAS_PER_SM 1
#endif
// Two CTAs per SM, each with its own ring: while one stops streaming (a segment's first threshold,
// a checkpoint, a hand-off) the other keeps its copies in flight, so the SM's HBM demand stays up.
constexpr int F_CPS = PB_STREAM_CTAS_PER_SM;  // resident CTAs per SM
constexpr int F_CW = 16 / F_CPS;            // consumer warps
constexpr int F_CT = F_CW * 32;             // consumer threads
constexpr int F_PROD = F_CW;                // producer warp
constexpr int F_NF = (F_CPS == 1) ? 2 : 1;  // finisher warps (segments alternate between them)
constexpr int F_NB = 2 * F_NF;              // list buffers (two per finisher)
constexpr int F_FIN = F_CW + 1;             // first finisher warp
constexpr int F_THREADS = (F_CW + 1 + F_NF) * 32;
constexpr int F_CHUNK = 32768 / F_CPS;      // bytes per staged chunk
constexpr int F_NSTAGE = 4;                 // 128 KB of copies in flight per SM
constexpr int F_RING = F_NSTAGE * F_CHUNK;
constexpr int F_LCAP = 512;                 // candidates one segment hands to the finisher
constexpr int F_KMAX = OFFER_PREFER;        // largest top_k settled here (thresholds from the offer bound)
constexpr int F_SMAX = 256;                 // survivors the finisher orders
constexpr int F_VSL = (F_CPS == 1) ? 8 : 7; // 16-byte vectors each consumer thread can hold as candidates
constexpr int F_CAND = F_VSL * F_CT * 16 + F_VSL * F_CT * 4;  // the vectors and their first element's index
constexpr int F_SMEM = F_RING + F_CAND + F_NB * F_LCAP * 8;
constexpr int F_SEGCAP = 128;               // segments whose mode the prologue caches in shared memory
constexpr int64_t F_RETRY = -2;             // out_token mark: the cluster kernel samples this row
constexpr int32_t F_CAND_RETRY = 0x400;     // the same mark in a shard record's flags
static_assert(F_CPS * (F_SMEM + 4096) <= 228 * 1024, "F_CPS CTAs per SM, with their static shared state");
static_assert((F_CHUNK / 16) % F_CT == 0, "a chunk splits evenly over the consumer threads");
static_assert(F_SMAX <= F_LCAP && F_LCAP % 32 == 0, "finisher layout");

enum : int { F_NONE = 0, F_GREEDY = 1, F_FILTER = 2 };

// What the streaming kernel does with a row (the cluster kernel uses the same test to skip it):
// rejected parameters, temperature-only and top-p-only rows, top_k above F_KMAX and bad uniforms
// go to the cluster kernel.
__device__ __forceinline__ int fast_mode(const pb_row_params& p, int64_t V) {
  const bool bad = !(p.temperature >= 0.0) || !(p.top_p > 0.0 && p.top_p <= 1.0) || p.top_k < 0;
  if (bad) return F_NONE;
  if (p.temperature == 0.0) return F_GREEDY;
  if (p.top_k > 0 && p.top_k <= F_KMAX && (int64_t)p.top_k < V && row_draw_ok(p))
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
  // balanced mode (workspace): the batch is cut into equal shares of 16-byte vectors, one per CTA,
  // so a row may be split over neighbouring CTAs; each piece of a split row publishes a record in
  // seg_rec and the piece that arrives last (row_cnt) merges them
  int32_t balanced;
  unsigned long long* row_cnt;  // per work item: arrival counter (CNT_MAGIC in the high word)
  uint8_t* seg_rec;             // records of split rows' pieces, indexed by row + CTA
};

// What the consumer warps hand a finisher for one segment, accumulated with shared-memory atomics
// (each warp adds its part) and reset by the finisher before it frees the buffer.
constexpr uint32_t LF_OVF = 1;  // a thread's candidate slots or the list overflowed
struct FastList {
  unsigned long long gcomp;  // greedy: largest composite (raw key, first index) over the warps
  uint32_t n;                // top-k: list entries the warps reserved (above F_LCAP: overflow)
  uint32_t maxkey;           // key of the segment's largest raw value (NaN above every key)
  uint32_t flags;            // LF_*
  uint32_t pad;
};

// ---- segments -------------------------------------------------------------------------------------
//
// Whole-row mode: CTA g takes rows g, g + grid, ... Balanced mode: the batch is a flat sequence of
// n_rows * U virtual vectors (U = ceil(vocab / EPV)); CTA g takes [g N / G, (g + 1) N / G) of it,
// which covers a piece of row `rf`, whole rows, and a piece of row `rl`. Only the first and the
// last segment of a CTA can be pieces. The CTA works on its last segment first and then the others
// in row order, so that both pieces of a row split between CTAs g and g + 1 are streamed at the
// start of the launch, and a CTA ends on a whole row when it has one. The host keeps every share
// at least SEG_MIN vectors long, so no CTA's share is empty.
constexpr int64_t SEG_MIN = 2048;                              // 32 KB
constexpr int F_SREC = 256;                                    // entries of a piece's record
constexpr unsigned long long CNT_MAGIC = 0xFFC0FFEEull << 32;  // a valid counter's high word

// The CTA's share, computed once (thread 0) so that no role divides 64-bit numbers per segment.
struct SegCta {
  int64_t A0, A1, U;
  int64_t rf, rl;
  int32_t count;                  // segments of this CTA
  int32_t nseg[2], first_rec[2];  // balanced mode: the pieces at segments 0 and 1
};

struct FastShared {
  uint64_t full[F_NSTAGE], empty[F_NSTAGE];  // ring: copy landed / every consumer warp done with it
  uint64_t lfull[F_NB], lfree[F_NB];         // list buffers: every consumer warp added / finisher done
  uint64_t cbar;                             // barrier of the consumer warps (count F_CW)
  uint64_t segready;                         // the producer warp has filled s_mk / s_tf
  int64_t issued[F_NSTAGE];                  // last chunk issued into each stage (-1: none)
  volatile int32_t abort;                    // a wait gave up: every role stops
  FastList lh[F_NB];
  SegCta sc;
  uint32_t s_mk[F_SEGCAP];  // per segment: mode << 30 | min(top_k, 2^30 - 1)
  float s_tf[F_SEGCAP];     // per segment: fp32(temperature)
  uint32_t cpb[2][F_CW];    // per checkpoint (alternating): each consumer warp's share of the offer bound
  uint32_t ob[F_CW];        // each consumer warp's share of a row's first threshold
  int32_t cp_flags[3];      // checkpoint flags (overflow 2, stop 4), rotating so a reset never races a write
  volatile int32_t pub[2];  // balanced mode: the piece at segment 0 / 1 has published its record
};

// Bounded wait that also gives up once another role has set `abort`.
__device__ __forceinline__ bool f_wait(uint64_t* bar, uint32_t parity, int limit, volatile int32_t* abort) {
  for (int i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
  }
  return false;
}

// Barrier of the consumer warps on an mbarrier (each warp's lane 0 arrives), with a bounded wait:
// a barrier that gives up returns false (and the CTA stops), so no warp can be left waiting on a
// barrier that another warp has stopped reaching. Orders the warps' shared-memory writes before
// it with their reads after it (arrive releases, the wait acquires).
__device__ __forceinline__ bool cbar_sync(FastShared& fs, uint32_t& phase) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&fs.cbar);
  const bool ok = __all_sync(0xFFFFFFFFu, f_wait(&fs.cbar, phase, WAIT_POLLS, &fs.abort));
  phase ^= 1;
  return ok;
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

struct FSeg {
  int64_t item;
  int64_t v0, v1;     // body vectors [v0, v1) of the row
  int64_t h_n, t_n;   // scalar head / tail elements this segment covers
  int32_t nseg;       // segments of the row (1: the whole row)
  int32_t first_rec;  // record index of the row's first piece (balanced mode)
  int32_t rec;        // this piece's record index
};

__device__ __forceinline__ int64_t seg_units(int64_t V, int epv) { return (V + epv - 1) / epv; }

// CTA whose share holds flat position P (the largest g with floor(g N / G) <= P).
__device__ __forceinline__ int64_t seg_cta_of(int64_t P, int64_t N, int64_t G) { return ((P + 1) * G - 1) / N; }

// The CTA's share (thread 0, once).
template <typename T>
__device__ void f_seg_cta(const FastArgs& a, SegCta* sc) {
  const int64_t G = gridDim.x, g = blockIdx.x;
  if (!a.balanced) {
    sc->A0 = sc->A1 = sc->U = sc->rf = sc->rl = 0;
    sc->count = (a.n_rows > g) ? (int32_t)((a.n_rows - g + G - 1) / G) : 0;
    sc->nseg[0] = sc->nseg[1] = 1;
    sc->first_rec[0] = sc->first_rec[1] = -1;
    return;
  }
  const int64_t U = seg_units(a.vocab, Elem<T>::EPV), N = a.n_rows * U;
  const int64_t A0 = g * N / G, A1 = (g + 1) * N / G;
  sc->A0 = A0;
  sc->A1 = A1;
  sc->U = U;
  sc->rf = A0 / U;
  sc->rl = (A1 - 1) / U;
  sc->count = (A1 > A0) ? (int32_t)(sc->rl - sc->rf + 1) : 0;
  for (int i = 0; i < 2; ++i) {
    const int64_t row = (i == 0) ? sc->rl : sc->rf;
    const int64_t gf = seg_cta_of(row * U, N, G), gl = seg_cta_of(row * U + U - 1, N, G);
    sc->nseg[i] = (int32_t)(gl - gf + 1);
    sc->first_rec[i] = (int32_t)(row + gf);
  }
}

// Work item of the CTA's i-th segment.
__device__ __forceinline__ int64_t f_seg_item(const FastArgs& a, const SegCta& sc, int i) {
  if (!a.balanced) return blockIdx.x + (int64_t)i * gridDim.x;
  return (i == 0) ? sc.rl : sc.rf + i - 1;
}

// The CTA's i-th segment (i < sc.count): no division.
template <typename T>
__device__ __forceinline__ void f_seg(const FastArgs& a, const SegCta& sc, int i, FSeg* s, FRow<T>* r) {
  const int64_t row = f_seg_item(a, sc, i);
  *r = f_row<T>(a, row);
  s->item = row;
  if (!a.balanced) {
    s->v0 = 0;
    s->v1 = r->nvec;
    s->h_n = r->head_n;
    s->t_n = r->tail_n;
    s->nseg = 1;
    s->first_rec = s->rec = -1;
    return;
  }
  const int64_t U = sc.U, base = row * U;
  const int64_t u0 = max(sc.A0, base) - base, u1 = min(sc.A1, base + U) - base;
  s->v0 = min(u0, r->nvec);
  s->v1 = min(u1, r->nvec);
  s->h_n = (u0 == 0) ? r->head_n : 0;
  s->t_n = (u1 == U) ? r->tail_n : 0;
  const bool whole = u0 == 0 && u1 == U;
  const int j = (i == 0) ? 0 : 1;  // (only segments 0 and 1 can be pieces)
  s->nseg = whole ? 1 : sc.nseg[j];
  s->first_rec = whole ? -1 : sc.first_rec[j];
  s->rec = (int32_t)(row + blockIdx.x);
}

// Mode (F_*), fp32 temperature and top_k of the CTA's i-th segment: cached by the prologue for the
// first F_SEGCAP segments, read from the parameters beyond.
__device__ __forceinline__ int f_seg_mode(const FastArgs& a, const FastShared& fs, int i, int64_t item, float* tf,
                                          int* k) {
  if (i < F_SEGCAP) {
    const uint32_t mk = fs.s_mk[i];
    *tf = fs.s_tf[i];
    *k = (int)(mk & 0x3FFFFFFFu);
    return (int)(mk >> 30);
  }
  const pb_row_params p = a.params[item];
  *tf = (float)p.temperature;
  *k = min(p.top_k, 0x3FFFFFFF);
  return fast_mode(p, a.vocab);
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
  FSeg sg;
  FRow<T> r;
  for (int i = 0; i < fs.sc.count; ++i) {
    float tf;
    int k;
    if (f_seg_mode(a, fs, i, f_seg_item(a, fs.sc, i), &tf, &k) == F_NONE) continue;
    f_seg<T>(a, fs.sc, i, &sg, &r);
    const int nvec = (int)(sg.v1 - sg.v0);
    const uint4* src = reinterpret_cast<const uint4*>(r.row + r.vec_e0) + sg.v0;
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
  warp_finish_sorted<NPL>(v, S, m, topp, (float)p.top_p, row_u53(p), &f);
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


// Cut a list of n <= 32 * NPL raw composites at L to the survivors of its kq largest: the exact
// kq-th largest raw key by bisection (always a key of the list), then every entry whose scaled key
// reaches the scaled kq-th key (x / T is monotone, so ties made by the division are kept: a raw
// value survives iff it is at or above the tie floor of the k-th). The survivors keep their raw
// composites, in list order, at L[0..return). All 32 lanes call.
template <int NPL>
__device__ int f_cut(uint64_t* L, int n, int kq, float tf) {
  const int lane = threadIdx.x & 31;
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
  // the largest X with #(keys >= X) >= kq; when exactly kq keys reach some mid, it is the smallest
  // of them
  uint32_t lo = mn;
  uint64_t hi = (uint64_t)mx + 1;
  while (hi - lo > 1) {
    const uint32_t mid = (uint32_t)(lo + ((hi - lo) >> 1));
    uint32_t cnt = 0, sm = 0xFFFFFFFFu;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      cnt += (kk[j] >= mid) ? 1u : 0u;
      sm = (kk[j] >= mid) ? min(sm, kk[j]) : sm;
    }
    cnt = __reduce_add_sync(0xFFFFFFFFu, cnt);
    if (cnt == (uint32_t)kq) {
      lo = __reduce_min_sync(0xFFFFFFFFu, sm);
      break;
    }
    if (cnt > (uint32_t)kq) lo = mid;
    else hi = mid;
  }
  const float lf = tie_floor(value_of(lo), tf);  // -inf: not an ordinary value; divide per entry
  const uint32_t lfk = key_of(lf);
  const uint32_t kth_s = key_of(__fdiv_rn(value_of(lo), tf));
  bool sv[NPL];
  int cnt = 0;
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    bool keep = j * 32 + lane < n && kk[j] >= lfk;
    if (lf == -INFINITY && keep) keep = kk[j] >= lo || key_of(__fdiv_rn(value_of(kk[j]), tf)) >= kth_s;
    sv[j] = keep;
    cnt += keep ? 1 : 0;
  }
  const int incl = warp_incl_scan(cnt);
  const int total = __shfl_sync(0xFFFFFFFFu, incl, 31);
  __syncwarp();  // every lane holds its list entries in registers: L may be overwritten
  int w = incl - cnt;
#pragma unroll
  for (int j = 0; j < NPL; ++j)
    if (sv[j]) L[w++] = c[j];
  __syncwarp();
  return total;
}

__device__ int f_cut_any(uint64_t* L, int n, int kq, float tf) {
  if (n <= 128) return f_cut<4>(L, n, kq, tf);
  if (n <= 256) return f_cut<8>(L, n, kq, tf);
  return f_cut<F_LCAP / 32>(L, n, kq, tf);
}

// Settle a top-k row from n <= F_LCAP raw composites at L that hold every survivor; m is the row's
// largest scaled key. Lists longer than two entries per lane are cut to the survivors first (a
// bisection costs far less than sorting the longer list). False: the row goes to the cluster kernel.
__device__ bool f_settle(const FastArgs& a, const pb_row_params& p, int64_t item, uint64_t* L, int n, float m) {
  if (n > 64) {
    n = f_cut_any(L, n, min(p.top_k, n), (float)p.temperature);
    if (n > F_SMAX) return false;
  }
  if (n <= 64) finish_list<2>(a, p, item, L, n, m);
  else if (n <= 128) finish_list<4>(a, p, item, L, n, m);
  else finish_list<8>(a, p, item, L, n, m);
  return true;
}

// Outputs of a row whose pieces report a timed-out wait.
__device__ void f_write_timeout(const FastArgs& a, int64_t item) {
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

// A greedy row's result: its first maximum (or index 0 when every value is -inf).
__device__ void f_write_greedy(const FastArgs& a, int64_t item, uint64_t comp) {
  const uint32_t idx = comp_idx(comp);
  const bool none = idx == 0xFFFFFFFFu;
  const float bestv = none ? -INFINITY : value_of(comp_key(comp));
  const uint32_t tok = none ? 0u : idx;
  if (a.cand_out) {
    uint8_t* rec = a.cand_out + item * record_bytes(a.cand_cap);
    reinterpret_cast<uint64_t*>(rec + sizeof(pb_cand_header))[0] = compose(key_of(bestv), tok + (uint32_t)a.vocab_offset);
    pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(rec);
    hd->count = 1;
    hd->flags = PB_CAND_GREEDY;
    hd->max_key = bestv;
    hd->reserved = 0;
    return;
  }
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

__device__ __forceinline__ uint8_t* f_rec(const FastArgs& a, int idx) {
  return a.seg_rec + (int64_t)idx * record_bytes(F_SREC);
}

// Arrival of one piece of a split row (lane 0; the piece's record is written): the row's token is
// marked for the cluster kernel first, so that a row whose merge never runs is still sampled; then
// the counter. A counter word without CNT_MAGIC in its high half (fresh or reused memory) counts
// as zero. True for the piece that arrives last, which resets the counter for the next launch.
__device__ bool f_arrive(const FastArgs& a, int64_t item, int nseg) {
  a.out_token[item] = F_RETRY;
  __threadfence();
  unsigned long long* cnt = a.row_cnt + item;
  unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(cnt), now;
  while (true) {
    now = (((old >> 32) << 32) == CNT_MAGIC ? old : CNT_MAGIC) + 1;
    const unsigned long long seen = atomicCAS(cnt, old, now);
    if (seen == old) break;
    old = seen;
  }
  const bool last = (int)(now & 0xFFFFFFFFull) >= nseg;
  if (last) {
    atomicExch(cnt, CNT_MAGIC);
    __threadfence();  // every piece's record is visible to the merge that follows
  }
  return last;
}

// Merge a split row from its pieces' records (raw composites: each piece's survivors, with their
// smallest key in the header's `reserved`; a greedy piece holds its first maximum). L (F_LCAP
// entries) is this warp's list buffer. Two rounds of loads, each with every load in flight at
// once: the headers, then every entry. All lanes call.
__device__ void f_merge_row(const FastArgs& a, const pb_row_params& p, int64_t item, int first_rec, int nseg,
                            bool greedy, uint64_t* L) {
  const int lane = threadIdx.x & 31;
  int32_t fl = 0, total = 0;
  float mraw = -INFINITY;
  uint64_t best = 0;
  int4 myh = make_int4(0, 0, 0, 0);  // header of record `lane`
  for (int j = lane; j < nseg; j += 32) {
    const int4 hv = __ldcg(reinterpret_cast<const int4*>(f_rec(a, first_rec + j)));
    if (j == lane) myh = hv;
    fl |= hv.y;
    total += hv.x;
    mraw = fmax_nan(mraw, __int_as_float(hv.z));
    if (greedy && hv.x > 0)
      best = max(best, (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(f_rec(a, first_rec + j) +
                                                                                      sizeof(pb_cand_header))));
  }
  fl = (int32_t)__reduce_or_sync(0xFFFFFFFFu, (uint32_t)fl);
  total = (int32_t)__reduce_add_sync(0xFFFFFFFFu, (uint32_t)total);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mraw = fmax_nan(mraw, __shfl_xor_sync(0xFFFFFFFFu, mraw, o));
    best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
  }
  if (fl & PB_ROW_TIMEOUT) {
    if (lane == 0) f_write_timeout(a, item);
    return;
  }
  if (fl & F_CAND_RETRY) return;  // (the token already holds the mark)
  if (greedy) {
    if (lane == 0) f_write_greedy(a, item, best ? best : compose(KEY_NEG_INF, 0xFFFFFFFFu));
    return;
  }
  const float tf = (float)p.temperature;
  const float m = __fdiv_rn(mraw, tf);
  const uint32_t mk = key_of(m);
  if (mk >= KEY_POS_INF || mk <= KEY_NEG_INF || total == 0 || total > F_LCAP) {
    if (lane == 0) a.out_token[item] = F_RETRY;  // (the cluster kernel reports or samples the row)
    return;
  }
  // a piece holding at least kq entries bounds the row's kq-th key from below (its smallest key):
  // keep the entries whose scaled key reaches the largest such bound (its tie floor on raw values)
  const int kq = min(p.top_k, total);
  uint32_t lb = 0;
  for (int j = lane; j < nseg; j += 32) {
    const int4 hv = (j == lane) ? myh : __ldcg(reinterpret_cast<const int4*>(f_rec(a, first_rec + j)));
    if (hv.x >= kq) lb = max(lb, (uint32_t)hv.w);
  }
  lb = __reduce_max_sync(0xFFFFFFFFu, lb);
  const uint32_t lbk = (lb > KEY_NEG_INF) ? key_of(tie_floor(value_of(lb), tf)) : 0u;
  // every entry into L (record j at the prefix of the counts before it)
  int base_off = 0;
  for (int g0 = 0; g0 < nseg; g0 += 32) {
    const int j = g0 + lane;
    const int cnt_l = (j >= nseg) ? 0 : (g0 == 0) ? myh.x : __ldcg(reinterpret_cast<const int*>(f_rec(a, first_rec + j)));
    const int incl = warp_incl_scan(cnt_l);
    const int ng = min(32, nseg - g0);
    for (int jj = 0; jj < ng; ++jj) {
      const int cnt = __shfl_sync(0xFFFFFFFFu, cnt_l, jj), off = base_off + __shfl_sync(0xFFFFFFFFu, incl, jj) - cnt;
      const unsigned long long* e =
          reinterpret_cast<const unsigned long long*>(f_rec(a, first_rec + g0 + jj) + sizeof(pb_cand_header));
      for (int i = lane; i < cnt; i += 32) L[off + i] = (uint64_t)__ldcg(e + i);
    }
    base_off += __shfl_sync(0xFFFFFFFFu, incl, 31);
  }
  __syncwarp();
  int n = 0;
  for (int base = 0; base < total; base += 32) {  // in place: every write lands at or below its read
    const int i = base + lane;
    const uint64_t v = (i < total) ? L[i] : 0ull;
    const bool keep = i < total && comp_key(v) >= lbk;
    const uint32_t bl = __ballot_sync(0xFFFFFFFFu, keep);
    __syncwarp();
    if (keep) L[n + __popc(bl & lanemask_lt())] = v;
    n += __popc(bl);
  }
  __syncwarp();
  if (!f_settle(a, p, item, L, n, m)) {
    if (lane == 0) a.out_token[item] = F_RETRY;
  }
}

// Publish one piece of a split row (its survivors with their smallest key, or a greedy piece's
// first maximum) and, when it is the row's last piece to arrive, merge the row. `retry`: the
// piece cannot describe its part.
__device__ void f_piece(const FastArgs& a, const pb_row_params& p, bool greedy, uint64_t gcomp, int n, bool retry,
                        float mraw, int seg, const FSeg& sg, uint64_t* L, volatile int32_t* pub) {
  const int lane = threadIdx.x & 31;
  uint8_t* rec = f_rec(a, sg.rec);
  uint64_t* ent = reinterpret_cast<uint64_t*>(rec + sizeof(pb_cand_header));
  uint32_t mn = 0xFFFFFFFFu;
  if (greedy) {
    n = (comp_idx(gcomp) != 0xFFFFFFFFu) ? 1 : 0;
    if (lane == 0 && n) ent[0] = gcomp;
  } else if (!retry) {
    if (n > p.top_k) n = f_cut_any(L, n, p.top_k, (float)p.temperature);
    if (n > F_SREC) {
      retry = true;
    } else {
      for (int i = lane; i < n; i += 32) {
        ent[i] = L[i];
        mn = min(mn, comp_key(L[i]));
      }
    }
    mn = __reduce_min_sync(0xFFFFFFFFu, mn);
  }
  bool last = false;
  if (lane == 0) {
    pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(rec);
    hd->count = retry ? 0 : n;
    hd->flags = retry ? F_CAND_RETRY : 0;
    hd->max_key = mraw;
    hd->reserved = (int32_t)((n > 0 && !retry && !greedy) ? mn : 0u);
    last = f_arrive(a, sg.item, sg.nseg);
    if (seg < 2) pub[seg] = 1;
  }
  __syncwarp();
  if (__shfl_sync(0xFFFFFFFFu, last ? 1 : 0, 0)) f_merge_row(a, p, sg.item, sg.first_rec, sg.nseg, greedy, L);
}

// One segment's result, from what the consumer warps accumulated in h (and, for top-k segments,
// the list L).
__device__ void f_segment(const FastArgs& a, const pb_row_params& p, int mode, const FastList& h, const FSeg& sg,
                          int seg, uint64_t* L, volatile int32_t* pub) {
  const int lane = threadIdx.x & 31;
  const float mraw = value_of(h.maxkey);
  if (mode == F_GREEDY) {
    const bool nan = h.maxkey == 0xFFFFFFFFu;  // a NaN: the cluster kernel finds the first one
    if (sg.nseg > 1) {
      f_piece(a, p, true, h.gcomp, 1, nan, mraw, seg, sg, L, pub);
    } else if (lane == 0) {
      if (nan) f_mark_retry(a, sg.item);
      else f_write_greedy(a, sg.item, h.gcomp);
    }
    return;
  }
  const bool ovf = (h.flags & LF_OVF) || h.n > (uint32_t)F_LCAP;
  if (sg.nseg > 1) {
    f_piece(a, p, false, 0, (int)h.n, ovf || h.maxkey >= KEY_POS_INF, mraw, seg, sg, L, pub);
    return;
  }
  const float m = __fdiv_rn(mraw, (float)p.temperature);
  const uint32_t mk = key_of(m);
  const bool retry = ovf || h.n == 0 || mk >= KEY_POS_INF || mk <= KEY_NEG_INF;
  if (retry || !f_settle(a, p, sg.item, L, (int)h.n, m)) {
    if (lane == 0) f_mark_retry(a, sg.item);
  }
}

template <typename T>
__device__ void f_finisher(const FastArgs& a, FastShared& fs, uint64_t* lists, int fin) {
  const int lane = threadIdx.x & 31;
  uint32_t lseq = 0;  // segments handed over so far (this warp takes every F_NF-th)
  FSeg sg;
  FRow<T> r;
  for (int i = 0; i < fs.sc.count; ++i) {
    float tf;
    int k;
    const int mode = f_seg_mode(a, fs, i, f_seg_item(a, fs.sc, i), &tf, &k);
    if (mode == F_NONE) continue;
    const uint32_t mine = lseq++;
    if ((int)(mine % F_NF) != fin) continue;
    f_seg<T>(a, fs.sc, i, &sg, &r);
    const pb_row_params p = a.params[sg.item];  // (in flight during the wait)
    const int b = (int)(mine % F_NB);
    if (!__all_sync(0xFFFFFFFFu, f_wait(&fs.lfull[b], (mine / F_NB) & 1, WAIT_POLLS, &fs.abort))) {
      if (lane == 0) fs.abort = 1;
      return;
    }
    FastList h;
    h.gcomp = fs.lh[b].gcomp;
    h.n = fs.lh[b].n;
    h.maxkey = fs.lh[b].maxkey;
    h.flags = fs.lh[b].flags;
    f_segment(a, p, mode, h, sg, i, lists + b * F_LCAP, fs.pub);
    __syncwarp();  // the list is read before the consumers may refill it
    if (lane == 0) {
      fs.lh[b].gcomp = 0;
      fs.lh[b].n = 0;
      fs.lh[b].maxkey = 0;
      fs.lh[b].flags = 0;
      mbar_arrive(&fs.lfree[b]);
    }
  }
}

// ---- consumers ------------------------------------------------------------------------------------

// The c-th largest of the warp's 32 keys (counted with multiplicity; 1 <= c <= 32): c rounds of a
// warp max, each taking one holder of the maximum out. Every lane gets it.
__device__ __forceinline__ uint32_t warp_cth_largest(uint32_t key, int c) {
  const int lane = threadIdx.x & 31;
  uint32_t m = 0;
  for (int r = 0; r < c; ++r) {
    m = __reduce_max_sync(0xFFFFFFFFu, key);
    const uint32_t holders = __ballot_sync(0xFFFFFFFFu, key == m);
    if (lane == __ffs(holders) - 1) key = 0;
  }
  return m;
}

// The offer bound of the consumer group: every thread offers one key (0: none); each warp sorts
// its 32 offers (bitonic, in registers) and publishes its ceil(k / F_CW)-th largest; the smallest
// over the warps is reached by at least k offers. Every thread gets the same key in *out. One
// barrier; `slot` must not be read by another call until a later barrier. False: the barrier gave up.
__device__ __forceinline__ bool f_offer_bound(uint32_t key, int k, uint32_t* slot, FastShared& fs, uint32_t& ph,
                                              uint32_t* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t kj = warp_cth_largest(key, (k + F_CW - 1) / F_CW);
  if (lane == 0) slot[warp] = kj;
  if (!cbar_sync(fs, ph)) return false;
  uint32_t mn = 0xFFFFFFFFu;
#pragma unroll
  for (int w = 0; w < F_CW; ++w) mn = min(mn, slot[w]);
  *out = mn;
  return true;
}

// Candidates of a top-k row are whole 16-byte vectors: a thread keeps (in shared memory) every
// vector of its own that holds a value at or above the threshold, with the index of its first
// element. Storing a vector costs no per-element work in the streaming loop; the values are
// looked at one by one only when the threshold rises and when the segment is handed off.

// Checkpoints of a segment (after chunk c): after 4 chunks (the first threshold, from one chunk, is
// loose), then every 12 chunks, and after the last chunk. In chunks, not bytes: a chunk gives every
// consumer thread the same number of vectors whatever the CTA's size, and it is that number the
// threads' candidate slots must absorb between checkpoints.
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
  constexpr int VPT = CV / F_CT;    // vectors per thread per chunk
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint4* vs = cand;                                                 // held vectors: slot j of thread t at j * F_CT + t
  uint32_t* vb = reinterpret_cast<uint32_t*>(cand + F_VSL * F_CT);  // index of each held vector's first element
  uint32_t seq = 0, lseq = 0, ph = 0;
  int cp = 0;         // checkpoints passed (their flag words rotate over three slots)
  bool stop = false;  // the CTA gave up (uniform over the consumers)
  FSeg sg;
  FRow<T> r;
  for (int si = 0; si < fs.sc.count && !stop; ++si) {
    float tf;
    int k;
    const int mode = f_seg_mode(a, fs, si, f_seg_item(a, fs.sc, si), &tf, &k);
    if (mode == F_NONE) continue;
    f_seg<T>(a, fs.sc, si, &sg, &r);
    const bool greedy = mode == F_GREEDY;
    const int nvec = (int)(sg.v1 - sg.v0);
    const int nch = (nvec + CV - 1) / CV;
    float runmax = -INFINITY, bestv = -INFINITY;
    uint32_t bidx = 0xFFFFFFFFu;
    int nc = 0;             // vectors this thread holds
    bool ovf = false;       // a vector of this thread found no free slot
    bool row_ovf = false;   // some thread overflowed (uniform: agreed at checkpoints)
    float t = -INFINITY;    // candidate threshold (a tie floor); changes only at barriers
    const uint32_t e_base = (uint32_t)(r.vec_e0 + sg.v0 * EPV) + (uint32_t)tid * EPV;  // element of vector tid of chunk 0
    for (int c = 0; c < nch; ++c, ++seq) {
      const int st = (int)(seq % F_NSTAGE);
      if (!__all_sync(0xFFFFFFFFu, f_wait(&fs.full[st], (seq / F_NSTAGE) & 1, a.poll_limit, &fs.abort))) {
        stop = true;
        break;
      }
      const int nv = min(CV, nvec - c * CV);
      const uint4* buf = ring + st * CV;
      // this thread's vectors of the chunk as raw words (-inf past the chunk's end)
      uint4 w[VPT];
      if (nv == CV) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) w[j] = buf[j * F_CT + tid];
      } else {
        const uint4 pad = make_uint4(E::NEG_INF_WORD, E::NEG_INF_WORD, E::NEG_INF_WORD, E::NEG_INF_WORD);
#pragma unroll
        for (int j = 0; j < VPT; ++j) w[j] = (j * F_CT + tid < nv) ? buf[j * F_CT + tid] : pad;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&fs.empty[st]);  // the vectors are in registers
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
        continue;
      }
      if (c == 0) {
        // first threshold: a lower bound of the segment's k-th value from this chunk (each warp's
        // ceil(k/16)-th largest per-thread maximum, the smallest over the warps), as a tie floor
        uint32_t lo = 0;
        if (nv * EPV >= k && !f_offer_bound(key_of(tm), k, fs.ob, fs, ph, &lo)) {  // nv is the same for all
          stop = true;
          break;
        }
        t = (lo > KEY_NEG_INF) ? tie_floor(value_of(lo), tf) : -INFINITY;  // (same in every thread)
      }
      if (!row_ovf && tm >= t) {
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
      if (f_checkpoint(c, nch)) {
        // checkpoint (one barrier): agree on overflow and stopping, and raise the threshold by the
        // offer bound of the values held (every thread offers its largest; each warp's
        // ceil(k/16)-th largest offer, the smallest over the warps, is reached by at least k of
        // them), then each thread drops its vectors below the new threshold
        float top = -INFINITY;
        for (int j = 0; j < nc; ++j) top = fmax_nan(top, vec_max<T>(vs[j * F_CT + tid]));
        const uint32_t kj = warp_cth_largest(nc > 0 ? key_of(top) : 0u, (k + F_CW - 1) / F_CW);
        const bool wovf = __any_sync(0xFFFFFFFFu, ovf);
        if (lane == 0) {
          fs.cpb[cp & 1][warp] = kj;
          const int mine = (fs.abort ? 4 : 0) | (wovf ? 2 : 0);
          if (mine) atomicOr(&fs.cp_flags[cp % 3], mine);
        }
        if (!cbar_sync(fs, ph)) {
          stop = true;
          break;
        }
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
    for (int64_t e = tid; e < sg.h_n + sg.t_n; e += F_CT) {
      const int64_t ei = (e < sg.h_n) ? e : r.tail_e0 + (e - sg.h_n);
      const float xv = E::ld(r.row + ei);
      runmax = fmax_nan(runmax, xv);
      if (greedy && (xv > bestv || (xv == bestv && (uint32_t)ei < bidx))) {
        bestv = xv;
        bidx = (uint32_t)ei;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) runmax = fmax_nan(runmax, __shfl_xor_sync(0xFFFFFFFFu, runmax, o));

    // hand the segment over: each warp adds its part to list buffer b on its own (the buffer is free
    // once its previous finisher released it) and arrives on its full barrier
    const int b = (int)(lseq % F_NB);
    FastList& lh = fs.lh[b];
    if (greedy) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xFFFFFFFFu, bestv, o);
        const uint32_t i2 = __shfl_xor_sync(0xFFFFFFFFu, bidx, o);
        if (v2 > bestv || (v2 == bestv && i2 < bidx)) {
          bestv = v2;
          bidx = i2;
        }
      }
      bool ok = true;
      if (lane == 0) {
        ok = f_wait(&fs.lfree[b], ((lseq / F_NB) & 1) ^ 1, WAIT_POLLS, &fs.abort);
        if (ok) {
          atomicMax(&lh.gcomp, (unsigned long long)compose(key_of(bestv), bidx));
          atomicMax(&lh.maxkey, key_of(runmax));
          mbar_arrive(&fs.lfull[b]);
        }
      }
      if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) {
        stop = true;
        break;
      }
      ++lseq;
      continue;
    }
    // top-k row: the values >= t of the held vectors (the last checkpoint raised t after the last
    // chunk) and of the scalar head and tail
    uint32_t cnt = 0;
    if (!row_ovf) {
      for (int j = 0; j < nc; ++j) {
        float x[EPV];
        E::unpack(vs[j * F_CT + tid], x);
#pragma unroll
        for (int q = 0; q < EPV; ++q) cnt += (x[q] >= t) ? 1u : 0u;
      }
      for (int64_t e = tid; e < sg.h_n + sg.t_n; e += F_CT) {
        const int64_t ei = (e < sg.h_n) ? e : r.tail_e0 + (e - sg.h_n);
        cnt += (E::ld(r.row + ei) >= t) ? 1u : 0u;
      }
    }
    const uint32_t incl = warp_incl_scan(cnt);
    const uint32_t wsum = __shfl_sync(0xFFFFFFFFu, incl, 31);
    bool ok = true;
    uint32_t base = 0;
    if (lane == 0) {
      ok = f_wait(&fs.lfree[b], ((lseq / F_NB) & 1) ^ 1, WAIT_POLLS, &fs.abort);
      if (ok) {
        base = atomicAdd(&lh.n, wsum);
        atomicMax(&lh.maxkey, key_of(runmax));
        if (row_ovf) atomicOr(&lh.flags, LF_OVF);
      }
    }
    if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) {
      stop = true;
      break;
    }
    base = __shfl_sync(0xFFFFFFFFu, base, 0);
    if (!row_ovf && base + wsum <= (uint32_t)F_LCAP) {
      uint64_t* L = lists + b * F_LCAP;
      uint32_t pos = base + incl - cnt;
      for (int j = 0; j < nc; ++j) {
        float x[EPV];
        E::unpack(vs[j * F_CT + tid], x);
        const uint32_t e0 = vb[j * F_CT + tid];
#pragma unroll
        for (int q = 0; q < EPV; ++q)
          if (x[q] >= t) L[pos++] = compose(key_of(x[q]), e0 + (uint32_t)q);
      }
      for (int64_t e = tid; e < sg.h_n + sg.t_n; e += F_CT) {
        const int64_t ei = (e < sg.h_n) ? e : r.tail_e0 + (e - sg.h_n);
        const float xv = E::ld(r.row + ei);
        if (xv >= t) L[pos++] = compose(key_of(xv), (uint32_t)ei);
      }
    }
    __syncwarp();  // the warp's entries are written (and its slots read) before it arrives
    if (lane == 0) mbar_arrive(&fs.lfull[b]);
    ++lseq;
  }
  if (stop && lane == 0) fs.abort = 1;
}

// ---- the kernel ------------------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(F_THREADS, F_CPS) stream_kernel(FastArgs a) {
  extern __shared__ __align__(128) unsigned char dyn[];
  __shared__ FastShared fs;
  uint4* ring = reinterpret_cast<uint4*>(dyn);
  uint4* cand = reinterpret_cast<uint4*>(dyn + F_RING);
  uint64_t* lists = reinterpret_cast<uint64_t*>(dyn + F_RING + F_CAND);
  const int tid = threadIdx.x, warp = tid >> 5;
  griddep_launch_dependents();  // the cluster kernel that follows may launch; it waits for this grid
  const int lane = tid & 31;
  if (tid == F_PROD * 32) {
    for (int s = 0; s < F_NSTAGE; ++s) {
      mbar_init(&fs.full[s], 1);
      mbar_init(&fs.empty[s], F_CW);
      fs.issued[s] = -1;
    }
    for (int b = 0; b < F_NB; ++b) {
      mbar_init(&fs.lfull[b], F_CW);
      mbar_init(&fs.lfree[b], 1);
      fs.lh[b].gcomp = 0;
      fs.lh[b].n = 0;
      fs.lh[b].maxkey = 0;
      fs.lh[b].flags = 0;
    }
    mbar_init(&fs.cbar, F_CW);
    mbar_init(&fs.segready, 1);
    for (int i = 0; i < 3; ++i) fs.cp_flags[i] = 0;
    fs.abort = 0;
    fs.pub[0] = fs.pub[1] = 0;
    f_seg_cta<T>(a, &fs.sc);
    fence_mbar_init();
  }
  __syncthreads();
  if (warp == F_PROD) {
    // the producer warp caches every segment's mode (one lane per segment, loads in flight
    // together), then lane 0 streams; the other roles start once the cache is filled
    const int ncache = min(fs.sc.count, F_SEGCAP);
    for (int i = lane; i < ncache; i += 32) {
      const pb_row_params p = a.params[f_seg_item(a, fs.sc, i)];
      fs.s_mk[i] = ((uint32_t)fast_mode(p, a.vocab) << 30) | (uint32_t)min(max(p.top_k, 0), 0x3FFFFFFF);
      fs.s_tf[i] = (float)p.temperature;
    }
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&fs.segready);
      f_producer<T>(a, fs, ring);
    }
    __syncwarp();  // (the warp reaches the CTA barrier below converged)
  } else if (__all_sync(0xFFFFFFFFu, f_wait(&fs.segready, 0, WAIT_POLLS, &fs.abort))) {
    if (warp >= F_FIN) f_finisher<T>(a, fs, lists, warp - F_FIN);
    else f_consumers<T>(a, fs, ring, cand, lists);
  } else if (lane == 0) {
    fs.abort = 1;
  }
  __syncthreads();
  if (fs.abort && tid == 0) {
    // let every issued copy land before the shared memory is released, then report the CTA's rows
    for (int s = 0; s < F_NSTAGE; ++s)
      if (fs.issued[s] >= 0) mbar_wait_bounded(&fs.full[s], (uint32_t)((fs.issued[s] / F_NSTAGE) & 1), WAIT_POLLS);
    FSeg sg;
    FRow<T> r;
    for (int i = 0; i < fs.sc.count; ++i) {
      float tf;
      int k;
      if (f_seg_mode(a, fs, i, f_seg_item(a, fs.sc, i), &tf, &k) == F_NONE) continue;
      f_seg<T>(a, fs.sc, i, &sg, &r);
      const int64_t item = sg.item;
      if (a.cand_out) {
        pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(a.cand_out + item * record_bytes(a.cand_cap));
        hd->count = 0;
        hd->flags = PB_ROW_TIMEOUT;
        hd->max_key = 0.0f;
        hd->reserved = 0;
      } else if (sg.nseg > 1) {
        // a piece that has not published yet still arrives (with a timed-out record), so that the
        // row's counter completes and its merge reports the timeout
        if (i < 2 && fs.pub[i]) continue;
        pb_cand_header* hd = reinterpret_cast<pb_cand_header*>(f_rec(a, sg.rec));
        hd->count = 0;
        hd->flags = PB_ROW_TIMEOUT;
        hd->max_key = 0.0f;
        hd->reserved = 0;
        if (f_arrive(a, item, sg.nseg)) f_write_timeout(a, item);
      } else {
        f_write_timeout(a, item);
      }
    }
  }
}
