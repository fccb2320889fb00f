// Two-pass sampler of the workspace path: a streaming pass that reduces every 128-byte group of the
// batch to the key of its largest value, then one CTA per row that settles greedy and small top-k
// rows from the few groups that can hold their survivors.
//
// Included by pb_sample.cu inside its anonymous namespace, after pb_stream.cuh: rows are settled
// with the streaming kernel's finisher (f_settle, f_write_greedy, f_mark_retry), in the same fixed
// arithmetic (pagedbatch/sampling.py:12-27 as stated in include/pagedbatch_b200.h), and the rows
// it does not take (fast_mode F_NONE) or cannot settle are left to the cluster kernel, which runs
// next on the same stream.
//
// Pass 1 (group_max_kernel) reads every byte of the batch exactly once and writes
// gmax[item][j] = the key of the largest value among elements [j * GE, (j + 1) * GE) of the row
// (GE = 128 bytes / element size; NaN above every key). Its warps take equal contiguous runs of
// "tasks" (4 groups, 512 bytes: one 16-byte vector per lane), GM_UNROLL tasks in flight per lane;
// no warp ever waits for another. Output: 1/32 of the input bytes, kept in L2 for pass 2.
//
// Pass 2 (group_settle_kernel), one CTA per row, after pass 1 (programmatic launch dependency):
//   greedy rows: the first group holding the row's largest key is re-read for its first maximum.
//   top-k rows (k <= F_KMAX): each of the 8 warps takes the ceil(k / 8)-th largest of its lanes'
//     largest group keys; the smallest of these, b, is reached by at least k group keys, so by at
//     least k values:
//     the k-th largest value is >= b, and every survivor (x / T ties values just below the k-th
//     one) is at or above the tie floor of b. The groups whose key reaches that floor are listed
//     per warp and re-read by the whole CTA; their values at or above it are the candidates,
//     settled exactly by f_settle in one warp.
// For rows longer than GS_MAXG groups, pass 2 reads runs of `coarse` consecutive groups as one.
// In shard mode (vocabulary-parallel, cand_out set) pass 2 writes each row's candidate record (its
// survivors with global indices, or its first maximum) exactly as the streaming kernel does.

#ifndef PB_GM_MINB
#define PB_GM_MINB 4
#endif
#ifndef PB_GM_UNROLL
#define PB_GM_UNROLL 8
#endif
#ifndef PB_GM_TPW
#define PB_GM_TPW 0
#endif
constexpr int GM_GB = 128;                    // bytes per group
constexpr int GM_GV = GM_GB / 16;             // 16-byte vectors per group
constexpr int GM_THREADS = 256;
constexpr int GM_WARPS = GM_THREADS / 32;
constexpr int GM_MINB = PB_GM_MINB;           // CTAs per SM pass 1 is compiled for
constexpr int GM_UNROLL = PB_GM_UNROLL;       // tasks each lane has in flight (128 KB per SM)
// tasks per warp in CTAs of a fixed size (0: one wave of equal shares, measured fastest on B200)
constexpr int GM_TPW = PB_GM_TPW;
constexpr int GS_THREADS = 256;
constexpr int GS_NW = GS_THREADS / 32;
constexpr int GS_NPT = 16;                    // (coarse) group keys per thread, in runs of 4
constexpr int GS_MAXG = GS_THREADS * GS_NPT;  // coarse groups a row is read as
constexpr int GS_WCAP = 128;                  // groups one warp re-reads (more: the cluster kernel)
constexpr int GS_RU = 4;                      // re-read vectors in flight per lane
static_assert(GM_GV == 8, "a group is one 8-lane part of a warp's 512-byte load");
static_assert(GS_NPT % 4 == 0, "group keys are loaded as 16-byte vectors");
static_assert((F_KMAX + GS_NW - 1) / GS_NW <= 32 * GS_NPT, "each warp holds enough group keys");

struct GroupArgs {
  const char* logits;
  int64_t n_rows, vocab, row_stride_bytes;
  const int32_t* row_index;
  const pb_row_params* params;
  int64_t* out_token;
  pb_row_info* out_info;
  uint32_t* gmax;  // [n_rows][ngs] group keys (the first ngr of each row written)
  int32_t ngr;     // groups per row: ceil(vocab / GE)
  int32_t ngs;     // row stride of gmax: ngr rounded up to a multiple of 4
  int32_t coarse;  // groups per coarse group in pass 2: ceil(ngr / GS_MAXG)
  int64_t ntasks;  // ceil(n_rows * ngr / 4); n_rows * ngs < 2^31
  // vocabulary-parallel shard mode: per-row candidate records instead of tokens (else null)
  uint8_t* cand_out;
  int32_t cand_cap;
  int64_t vocab_offset;
};

__device__ __forceinline__ uint4 ld_once16(const void* p, uint64_t pol) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ void st_keep_u32(uint32_t* p, uint32_t v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.u32 [%0], %1, %2;" ::"l"(p), "r"(v), "l"(pol) : "memory");
}

// The n (< EPV) elements at p as a 16-byte vector, the missing ones -inf (below every element's
// key, so a group's largest key is unchanged).
template <typename T>
__device__ __noinline__ uint4 part_vec(const T* p, int n) {
  constexpr int EPV = Elem<T>::EPV;
  uint32_t w[4] = {Elem<T>::NEG_INF_WORD, Elem<T>::NEG_INF_WORD, Elem<T>::NEG_INF_WORD, Elem<T>::NEG_INF_WORD};
#pragma unroll
  for (int q = 0; q < EPV; ++q) {
    if (q < n) {
      if constexpr (EPV == 4) {
        w[q] = __ldg(reinterpret_cast<const uint32_t*>(p) + q);
      } else {
        const uint32_t b = __ldg(reinterpret_cast<const unsigned short*>(p) + q);
        const int sh = (q & 1) * 16;
        w[q >> 1] = (w[q >> 1] & ~(0xFFFFu << sh)) | (b << sh);
      }
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
__global__ void __launch_bounds__(GM_THREADS, GM_MINB) group_max_kernel(GroupArgs g) {
  constexpr int ES = Elem<T>::ES, EPV = Elem<T>::EPV, GE = GM_GB / ES;
  const int lane = threadIdx.x & 31, sub = lane >> 3, part = lane & 7;
  const int64_t W = (int64_t)gridDim.x * GM_WARPS;
  const int64_t w = (int64_t)blockIdx.x * GM_WARPS + (threadIdx.x >> 5);
  const int32_t ngr = g.ngr, ngs = g.ngs, nrows = (int32_t)g.n_rows, V = (int32_t)g.vocab;
  const uint64_t pol_in = l2_policy_evict_first(), pol_out = l2_policy_evict_last();
  // let pass 2 launch now: its CTAs take the SMs this pass frees and wait (griddepcontrol.wait)
  // until the whole pass has finished and its stores are visible
  griddep_launch_dependents();
  const int64_t t0 = w * g.ntasks / W, t1 = (w + 1) * g.ntasks / W;
  // this lane's group of task t is 4 t + sub: (row, j), advanced by 4 groups per task
  const int64_t gid = 4 * t0 + sub;
  int32_t row = (int32_t)(gid / ngr), j = (int32_t)(gid - (int64_t)row * ngr);
  int32_t cur = -1;
  const char* base = nullptr;
  for (int64_t t = t0; t < t1; t += GM_UNROLL) {
    uint4 v[GM_UNROLL];
    int32_t at[GM_UNROLL];  // gmax index of the lane's group, or -1
#pragma unroll
    for (int u = 0; u < GM_UNROLL; ++u) {
      at[u] = -1;
      v[u] = make_uint4(0u, 0u, 0u, 0u);
      if (t + u < t1 && row < nrows) {
        if (row != cur) {
          cur = row;
          base = g.logits + (g.row_index ? (int64_t)g.row_index[row] : (int64_t)row) * g.row_stride_bytes;
        }
        at[u] = row * ngs + j;
        const int32_t e0 = j * GE + part * EPV;
        if (e0 + EPV <= V) v[u] = ld_once16(base + (int64_t)e0 * ES, pol_in);
        else v[u] = part_vec<T>(reinterpret_cast<const T*>(base) + e0, V - e0);  // empty: every element -inf
      }
      j += 4;
      while (j >= ngr) {
        j -= ngr;
        ++row;
      }
    }
#pragma unroll
    for (int u = 0; u < GM_UNROLL; ++u) {
      uint32_t k = key_of(vec_max<T>(v[u]));
      k = max(k, __shfl_xor_sync(0xFFFFFFFFu, k, 1));
      k = max(k, __shfl_xor_sync(0xFFFFFFFFu, k, 2));
      k = max(k, __shfl_xor_sync(0xFFFFFFFFu, k, 4));
      if (part == 0 && at[u] >= 0) st_keep_u32(g.gmax + at[u], k, pol_out);
    }
  }
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = max(x, __shfl_xor_sync(0xFFFFFFFFu, x, o));
  return x;
}

// Candidates of the CTA's listed groups: warp w listed cnt[w] coarse groups (R groups each) at
// lists + w * GS_WCAP; their 16-byte vectors are spread over all the CTA's threads, GS_RU per thread
// in flight. Every value at or above thr_v (the value of the threshold key; the row holds no NaN)
// goes to L (shared counter *n; entries past F_LCAP are counted, not stored). A vector whose largest
// value is below thr_v is skipped whole.
template <typename T>
__device__ __forceinline__ void cta_candidates(const T* row, const uint32_t* lists, const uint32_t* cnt, int32_t R,
                                               int64_t V, float thr_v, uint64_t* L, uint32_t* n) {
  constexpr int EPV = Elem<T>::EPV, GE = GM_GB / Elem<T>::ES;
  const uint32_t vpg = (uint32_t)R * GM_GV;
  uint32_t start[GS_NW + 1];
  start[0] = 0;
#pragma unroll
  for (int w = 0; w < GS_NW; ++w) start[w + 1] = start[w] + cnt[w] * vpg;
  const uint32_t nv = start[GS_NW];
  for (uint32_t b0 = 0; b0 < nv; b0 += GS_THREADS * GS_RU) {
    uint4 vv[GS_RU];
    int64_t ee[GS_RU];
#pragma unroll
    for (int u = 0; u < GS_RU; ++u) {
      const uint32_t vi = b0 + (uint32_t)(u * GS_THREADS + threadIdx.x);
      ee[u] = -1;
      vv[u] = make_uint4(0u, 0u, 0u, 0u);
      if (vi < nv) {
        int w = 0;
        uint32_t first = 0;
#pragma unroll
        for (int x = 1; x < GS_NW; ++x) {
          if (vi >= start[x]) {
            w = x;
            first = start[x];
          }
        }
        const uint32_t r = vi - first;  // vector r of warp w's list
        const uint32_t gsel = (R == 1) ? (r >> 3) : r / vpg;
        const uint32_t part = r - gsel * vpg;
        const int64_t e = (int64_t)lists[w * GS_WCAP + gsel] * R * GE + (int64_t)part * EPV;
        if (e < V) {
          ee[u] = e;
          vv[u] = (e + EPV <= V) ? *reinterpret_cast<const uint4*>(row + e) : part_vec<T>(row + e, (int)(V - e));
        }
      }
    }
    // this thread's candidates: a bit per element of each vector; one shared atomic per warp
    uint32_t mask[GS_RU];
    uint32_t mine = 0;
#pragma unroll
    for (int u = 0; u < GS_RU; ++u) {
      mask[u] = 0;
      if (ee[u] >= 0 && vec_max<T>(vv[u]) >= thr_v) {
        float x[EPV];
        Elem<T>::unpack(vv[u], x);
#pragma unroll
        for (int q = 0; q < EPV; ++q)
          if (x[q] >= thr_v && ee[u] + q < V) mask[u] |= 1u << q;
      }
      mine += (uint32_t)__popc(mask[u]);
    }
    const uint32_t incl = warp_incl_scan(mine);
    uint32_t base = 0;
    if ((threadIdx.x & 31) == 31 && incl) base = atomicAdd(n, incl);
    base = __shfl_sync(0xFFFFFFFFu, base, 31) + incl - mine;
#pragma unroll
    for (int u = 0; u < GS_RU; ++u) {
      while (mask[u]) {
        const int q = __ffs(mask[u]) - 1;
        mask[u] &= mask[u] - 1;
        if (base < (uint32_t)F_LCAP) L[base] = compose(key_of(Elem<T>::elem(vv[u], q)), (uint32_t)(ee[u] + q));
        ++base;
      }
    }
  }
}

// MINB: CTAs per SM the kernel is compiled for (2 for batches of up to two rows per SM; 4 for more
// rows, which then take fewer waves).
template <typename T, int MINB>
__global__ void __launch_bounds__(GS_THREADS, MINB) group_settle_kernel(GroupArgs g) {
  constexpr int EPV = Elem<T>::EPV, GE = GM_GB / Elem<T>::ES;
  __shared__ uint64_t L[F_LCAP];
  __shared__ uint32_t s_list[GS_NW * GS_WCAP];
  __shared__ uint32_t s_bound[GS_NW], s_max[GS_NW], s_cnt[GS_NW];
  __shared__ unsigned long long s_best[GS_NW];
  __shared__ uint32_t s_n;

  const int64_t item = blockIdx.x;
  const int64_t V = g.vocab;
  const pb_row_params p = g.params[item];
  const int mode = fast_mode(p, V);
  if (mode == F_NONE) return;  // the cluster kernel samples this row
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) s_n = 0;
  FastArgs fa;
  fa.logits = g.logits;
  fa.n_rows = g.n_rows;
  fa.vocab = V;
  fa.row_stride = 0;
  fa.row_index = g.row_index;
  fa.params = g.params;
  fa.out_token = g.out_token;
  fa.out_info = g.out_info;
  fa.cand_out = g.cand_out;
  fa.cand_cap = g.cand_cap;
  fa.vocab_offset = g.vocab_offset;
  fa.poll_limit = 0;
  fa.balanced = 0;
  fa.row_cnt = nullptr;
  fa.seg_rec = nullptr;
  const T* row = reinterpret_cast<const T*>(
      g.logits + (g.row_index ? (int64_t)g.row_index[item] : item) * g.row_stride_bytes);
  const int32_t ngr = g.ngr, R = g.coarse;
  const int32_t nc = (ngr + R - 1) / R;
  // this thread's coarse groups: runs of 4, the CTA's threads side by side, so every warp holds keys
  // from the whole row
  auto cidx = [&](int i) -> int32_t { return ((i >> 2) * GS_THREADS + tid) * 4 + (i & 3); };
  griddep_wait();  // pass 1's group keys
  const uint32_t* gm = g.gmax + item * (int64_t)g.ngs;
  uint32_t val[GS_NPT];
  if (R == 1) {
    // 16-byte loads of the row's keys (its stride is a multiple of 4 keys); keys past ngr are 0
#pragma unroll
    for (int i = 0; i < GS_NPT; i += 4) {
      uint4 q = make_uint4(0u, 0u, 0u, 0u);
      if (cidx(i) < ngr) q = __ldcg(reinterpret_cast<const uint4*>(gm + cidx(i)));
      val[i] = q.x;
      val[i + 1] = q.y;
      val[i + 2] = q.z;
      val[i + 3] = q.w;
    }
#pragma unroll
    for (int i = 0; i < GS_NPT; ++i)
      if (cidx(i) >= nc) val[i] = 0;
  } else {
#pragma unroll
    for (int i = 0; i < GS_NPT; ++i) {
      const int32_t c = cidx(i);
      uint32_t x = 0;
      if (c < nc) {
        const int32_t e = min(ngr, (c + 1) * R);
        for (int32_t gi = c * R; gi < e; ++gi) x = max(x, __ldcg(gm + gi));
      }
      val[i] = x;
    }
  }

  if (mode == F_GREEDY) {
    // the largest key and the first coarse group holding it (compose: index ascending on ties)
    unsigned long long best = 0;
#pragma unroll
    for (int i = 0; i < GS_NPT; ++i)
      if (cidx(i) < nc) best = max(best, (unsigned long long)compose(val[i], (uint32_t)cidx(i)));
    best = warp_max_u64(best);
    if (lane == 0) s_best[warp] = best;
    __syncthreads();
    if (warp != 0) return;
    best = 0;
#pragma unroll
    for (int w = 0; w < GS_NW; ++w) best = max(best, s_best[w]);
    const uint32_t mk = comp_key(best);
    if (mk == 0xFFFFFFFFu) {  // a NaN: the cluster kernel finds the first one
      if (lane == 0) f_mark_retry(fa, item);
      return;
    }
    const int64_t cb = comp_idx(best);
    const int64_t e_end = min(V, (cb + 1) * R * GE);
    uint32_t first = 0xFFFFFFFFu;
    for (int64_t e0 = cb * R * GE + (int64_t)lane * EPV; e0 < e_end; e0 += 32 * EPV) {
      const int n = (int)min((int64_t)EPV, V - e0);
      const uint4 vv = (n == EPV) ? *reinterpret_cast<const uint4*>(row + e0) : part_vec<T>(row + e0, n);
      float x[EPV];
      Elem<T>::unpack(vv, x);
#pragma unroll
      for (int q = 0; q < EPV; ++q)
        if (q < n && key_of(x[q]) == mk) first = min(first, (uint32_t)(e0 + q));
    }
    first = __reduce_min_sync(0xFFFFFFFFu, first);
    if (lane == 0) f_write_greedy(fa, item, compose(mk, first));
    return;
  }

  // top-k: the warp's cw-th largest lane maximum (each lane maximum is a group key, so at least cw of
  // the warp's group keys reach it); padding keys are 0, below every key
  const int cw = (p.top_k + GS_NW - 1) / GS_NW;
  uint32_t lm = 0;
#pragma unroll
  for (int i = 0; i < GS_NPT; ++i) lm = max(lm, val[i]);
  const uint32_t wmax = __reduce_max_sync(0xFFFFFFFFu, lm);
  const uint32_t kth = warp_cth_largest(lm, cw);
  if (lane == 0) {
    s_bound[warp] = kth;
    s_max[warp] = wmax;
  }
  __syncthreads();
  uint32_t bound = 0xFFFFFFFFu, rmax = 0;
#pragma unroll
  for (int w = 0; w < GS_NW; ++w) {
    bound = min(bound, s_bound[w]);
    rmax = max(rmax, s_max[w]);
  }
  const float tf = (float)p.temperature;
  const float m = __fdiv_rn(value_of(rmax), tf);
  const uint32_t mk = key_of(m);
  if (mk >= KEY_POS_INF || mk <= KEY_NEG_INF) {  // +inf or NaN values, or only -inf: the cluster kernel
    if (tid == 0) f_mark_retry(fa, item);
    return;
  }
  const uint32_t thr = (bound > KEY_NEG_INF) ? key_of(tie_floor(value_of(bound), tf)) : 0u;

  // each warp lists its lanes' groups whose key reaches thr; then the CTA re-reads them together
  uint32_t* wl = s_list + warp * GS_WCAP;
  uint32_t cnt = 0;
#pragma unroll
  for (int i = 0; i < GS_NPT; ++i) {
    const bool hit = cidx(i) < nc && val[i] >= thr;
    const uint32_t b = __ballot_sync(0xFFFFFFFFu, hit);
    const uint32_t pos = cnt + (uint32_t)__popc(b & lanemask_lt());
    if (hit && pos < (uint32_t)GS_WCAP) wl[pos] = (uint32_t)cidx(i);
    cnt += (uint32_t)__popc(b);
  }
  if (lane == 0) s_cnt[warp] = cnt;
  __syncthreads();
  bool over = false;
#pragma unroll
  for (int w = 0; w < GS_NW; ++w) over |= s_cnt[w] > (uint32_t)GS_WCAP;
  if (over) {  // more groups than the lists hold: the cluster kernel
    if (tid == 0) f_mark_retry(fa, item);
    return;
  }
  cta_candidates<T>(row, s_list, s_cnt, R, V, thr ? value_of(thr) : -INFINITY, L, &s_n);
  __syncthreads();
  const uint32_t n = s_n;
  if (warp != 0) return;
  if (n == 0 || n > (uint32_t)F_LCAP || !f_settle(fa, p, item, L, (int)n, m)) {
    if (lane == 0) f_mark_retry(fa, item);
  }
}
