/*
 * TEST INFRASTRUCTURE — CPU oracle for the pagedbatch sampling path. Only tests/, the
 * smoke() check and bench.py's cpu_baseline leg load this file's library; the product
 * (pagedbatch_b200) never does.
 *
 * A plain, sequential C restatement of pagedbatch/sampling.py:10-27 (sample_token) in the
 * exact arithmetic the B200 kernels implement:
 *   - greedy (temperature == 0, config.py:156-158): argmax of the raw row, NaN counts as the
 *     largest value and ties go to the lowest index (torch.argmax, sampling.py:13);
 *   - keys = fp32(x) / fp32(temperature), IEEE division (sampling.py:14);
 *   - top-k (0 < k < V): keep every key >= the k-th largest, ties included (sampling.py:15-17);
 *   - top-p (top_p < 1): sort keys descending (ties by index ascending), keep a position while
 *     the mass strictly before it is <= top_p of the total (sampling.py:18-25). Mass is the
 *     fixed-point weight q = floor(E(key - max) * 2^40), summed exactly in 64 bits;
 *   - draw: inverse CDF over the kept set in the same order with target
 *     floor(U53 * kept_mass / 2^53), U53 = uniform * 2^53 (the reference draws with
 *     torch.multinomial, sampling.py:26-27; see the parity notes in the tests).
 * E is a fixed exp: Cody-Waite reduction by ln2 (two-part constant) and the degree-7 Taylor
 * polynomial of e^r on |r| <= ln2/2, evaluated with explicit fmaf in a fixed order so that
 * this file and the device code produce the same bits. Build with -ffp-contract=off.
 *
 * Parity is pinned against fixtures produced by running the reference itself
 * (tests/golden/make_golden.py); this file does not read the reference.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/pagedbatch_b200.h"

/* ------------------------------------------------------------------------------------------ */
/* keys and the fixed exp                                                                       */
/* ------------------------------------------------------------------------------------------ */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* order-preserving key: NaN above everything (torch sorts NaN as largest), -0 folded onto +0 */
uint32_t pbo_key(float x) {
  if (x != x) return 0xFFFFFFFFu;
  uint32_t b = (x == 0.0f) ? 0u : f2u(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

float pbo_key_value(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return u2f(b);
}

float pbo_exp(float d) {
  if (!(d >= -87.0f)) return 0.0f;
  volatile float t = d * 0x1.715476p+0f;          /* log2(e) */
  float n = nearbyintf(t);                         /* round half to even */
  float r = fmaf(-n, 0x1.62e43p-1f, d);            /* ln2 high part */
  r = fmaf(-n, -0x1.05c61p-29f, r);                /* ln2 low part */
  float p = 0x1.a01a02p-13f;                       /* 1/7! */
  p = fmaf(p, r, 0x1.6c16c2p-10f);                 /* 1/6! */
  p = fmaf(p, r, 0x1.111112p-7f);                  /* 1/5! */
  p = fmaf(p, r, 0x1.555556p-5f);                  /* 1/4! */
  p = fmaf(p, r, 0x1.555556p-3f);                  /* 1/3! */
  p = fmaf(p, r, 0x1.0p-1f);                       /* 1/2! */
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int32_t ni = (int32_t)n;
  return u2f((uint32_t)((int32_t)f2u(p) + (ni << 23)));
}

static uint64_t weight_q(float key, float m) {
  float d = key - m;
  float w = pbo_exp(d);
  return (uint64_t)(w * 0x1p40f);
}

/* floor(p * z) for an fp32 p in [0, 1) and z < 2^64, exact */
static uint64_t mul_floor(float p, uint64_t z) {
  uint32_t b = f2u(p);
  uint32_t e8 = (b >> 23) & 0xFF;
  uint64_t man = b & 0x7FFFFF;
  int shift;
  if (e8 == 0) { shift = 149; } else { man |= 0x800000; shift = 150 - (int)e8; }
  if (shift >= 128 || man == 0) return 0;
  unsigned __int128 prod = (unsigned __int128)man * z;
  return (uint64_t)(prod >> shift);
}

static int load_row(const void* logits, int dtype, int64_t row, int64_t V, int64_t stride, float* x) {
  if (dtype == PB_DTYPE_F32) {
    const float* p = (const float*)logits + row * stride;
    memcpy(x, p, (size_t)V * 4);
  } else if (dtype == PB_DTYPE_BF16) {
    const uint16_t* p = (const uint16_t*)logits + row * stride;
    for (int64_t j = 0; j < V; j++) x[j] = u2f((uint32_t)p[j] << 16);
  } else if (dtype == PB_DTYPE_F16) {
    const uint16_t* p = (const uint16_t*)logits + row * stride;
    for (int64_t j = 0; j < V; j++) {
      uint32_t h = p[j], s = (h & 0x8000u) << 16, e = (h >> 10) & 0x1F, m = h & 0x3FF, out;
      if (e == 0) {
        if (m == 0) out = s;
        else { /* subnormal half: value m * 2^-24, exact in fp32 */
          float v = (float)m * 0x1p-24f;
          out = s | f2u(v);
        }
      } else if (e == 31) out = s | 0x7F800000u | (m << 13);
      else out = s | ((e + 112) << 23) | (m << 13);
      x[j] = u2f(out);
    }
  } else {
    return -1;
  }
  return 0;
}

/* sort order: key descending, index ascending */
typedef struct { uint32_t k; uint32_t i; } ent_t;

/* Philox4x32-10 as published (Salmon, Moraes, Dror, Shaw, SC 2011): per round the counter words
 * (c0, c1, c2, c3) become (hi(M1*c2) ^ c1 ^ k0, lo(M1*c2), hi(M0*c0) ^ c3 ^ k1, lo(M0*c0)) with
 * M0 = 0xD2511F53 and M1 = 0xCD9E8D57; the key is bumped by (0x9E3779B9, 0xBB67AE85) before every
 * round but the first. Checked against the algorithm's published known-answer vectors. */
void pbo_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t x[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
  uint32_t k[2] = {key[0], key[1]};
  for (int round = 0; round < 10; round++) {
    if (round) { k[0] += 0x9E3779B9u; k[1] += 0xBB67AE85u; }
    uint64_t a = (uint64_t)0xD2511F53u * x[0];
    uint64_t b = (uint64_t)0xCD9E8D57u * x[2];
    uint32_t y0 = (uint32_t)(b >> 32) ^ x[1] ^ k[0];
    uint32_t y2 = (uint32_t)(a >> 32) ^ x[3] ^ k[1];
    x[0] = y0; x[1] = (uint32_t)b; x[2] = y2; x[3] = (uint32_t)a;
  }
  memcpy(out, x, sizeof x);
}

/* The row's draw as U53 (pagedbatch_b200.h, pb_row_params.rng): the host uniform * 2^53, or for
 * PB_RNG_PHILOX rows Philox with key = the 64-bit seed stored in `uniform`'s bits and counter
 * (step, 0, 0, 0), U53 = (out[0] >> 11) << 32 | out[1]. Returns 0 when a host uniform is outside
 * [0, 1). */
int pbo_row_u53(const pb_row_params* prm, uint64_t* u53) {
  if (prm->rng & PB_RNG_PHILOX) {
    uint64_t seed;
    memcpy(&seed, &prm->uniform, 8);
    uint32_t ctr[4] = {prm->rng & 0x7FFFFFFFu, 0, 0, 0}, key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)}, o[4];
    pbo_philox4x32_10(ctr, key, o);
    *u53 = ((uint64_t)(o[0] >> 11) << 32) | o[1];
    return 1;
  }
  const double u = prm->uniform;
  if (!(u >= 0.0 && u < 1.0)) return 0;
  *u53 = (uint64_t)(u * 0x1p53);
  return 1;
}
static int ent_cmp(const void* a, const void* b) {
  const ent_t* x = (const ent_t*)a; const ent_t* y = (const ent_t*)b;
  if (x->k != y->k) return x->k > y->k ? -1 : 1;
  return x->i < y->i ? -1 : (x->i > y->i);
}

/* ------------------------------------------------------------------------------------------ */
/* one row                                                                                      */
/* ------------------------------------------------------------------------------------------ */

static void sample_row(const float* x, int64_t V, const pb_row_params* prm, ent_t* ent,
                       int64_t* tok, pb_row_info* info, float* probs) {
  pb_row_info inf;
  memset(&inf, 0, sizeof inf);
  if (probs) memset(probs, 0, (size_t)V * 4);

  /* values SamplingParams rejects (config.py:146-155) */
  if (!(prm->temperature >= 0.0) || !(prm->top_p > 0.0 && prm->top_p <= 1.0) || prm->top_k < 0) {
    inf.status = PB_ROW_BAD_PARAMS;
    *tok = -1;
    if (info) *info = inf;
    return;
  }

  if (prm->temperature == 0.0) {                   /* greedy: sampling.py:12-13 */
    uint32_t bk = 0; int64_t bi = 0;
    for (int64_t j = 0; j < V; j++) {
      uint32_t k = pbo_key(x[j]);
      if (j == 0 || k > bk) { bk = k; bi = j; }
    }
    inf.thr_key = bk; inf.n_tie_kept = 1; inf.kept_count = 1;
    inf.max_key = x[bi]; inf.flags = PB_PATH_GREEDY;
    *tok = bi;
    if (info) *info = inf;
    if (probs) probs[bi] = 1.0f;
    return;
  }

  const float tf = (float)prm->temperature;
  for (int64_t j = 0; j < V; j++) {                /* sampling.py:14 */
    volatile float y = x[j] / tf;
    ent[j].k = pbo_key(y);
    ent[j].i = (uint32_t)j;
  }
  qsort(ent, (size_t)V, sizeof(ent_t), ent_cmp);
  const uint32_t mk = ent[0].k;
  const float m = pbo_key_value(mk);
  inf.max_key = m;
  if (mk >= 0xFF800000u || mk <= 0x007FFFFFu) {   /* +inf / NaN max, or all -inf */
    inf.status = PB_ROW_NONFINITE; *tok = -1;
    if (info) *info = inf;
    return;
  }
  uint64_t u53;
  if (!pbo_row_u53(prm, &u53)) {
    inf.status = PB_ROW_BAD_UNIFORM; *tok = -1;
    if (info) *info = inf;
    return;
  }

  /* top-k: sampling.py:15-17 — every key >= the k-th largest survives */
  int64_t nk = V;
  const int32_t k = prm->top_k;
  if (k > 0 && (int64_t)k < V) {
    uint32_t kth = ent[k - 1].k;
    nk = k;
    while (nk < V && ent[nk].k >= kth) nk++;
  }

  uint64_t zq = 0;
  for (int64_t p = 0; p < nk; p++) zq += weight_q(pbo_key_value(ent[p].k), m);

  /* top-p: sampling.py:18-25 — keep position p while the mass before it is <= top_p * total */
  int64_t last = nk - 1;
  uint64_t kept = zq;
  const float pf = (float)prm->top_p;
  if (prm->top_p < 1.0 && pf < 1.0f) {
    uint64_t tp = mul_floor(pf, zq);
    uint64_t run = 0;
    for (int64_t p = 0; p < nk; p++) {
      run += weight_q(pbo_key_value(ent[p].k), m);
      if (run > tp) { last = p; kept = run; break; }
    }
  }

  /* draw: inverse CDF over the kept prefix (replaces torch.multinomial, sampling.py:27) */
  uint64_t t = (uint64_t)(((unsigned __int128)u53 * kept) >> 53);
  uint64_t run = 0;
  int64_t pick = last;
  for (int64_t p = 0; p <= last; p++) {
    run += weight_q(pbo_key_value(ent[p].k), m);
    if (run > t) { pick = p; break; }
  }
  *tok = ent[pick].i;

  int64_t first = last;
  while (first > 0 && ent[first - 1].k == ent[last].k) first--;
  inf.thr_key = ent[last].k;
  inf.n_tie_kept = (int32_t)(last - first + 1);
  inf.kept_count = (int32_t)(last + 1);
  inf.z_q = zq;
  inf.kept_q = kept;
  inf.flags = 0;
  if (info) *info = inf;

  if (probs) {                                     /* sampling.py:26 — softmax over the kept set */
    volatile float zf = (float)kept;
    zf = zf * 0x1p-40f;
    for (int64_t p = 0; p <= last; p++) {
      float w = pbo_exp(pbo_key_value(ent[p].k) - m);
      probs[ent[p].i] = w / zf;
    }
  }
}

int pbo_sample(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
               const int32_t* row_index, const pb_row_params* params, int64_t* out_token,
               pb_row_info* out_info, float* out_probs) {
  if (!logits || !params || !out_token || vocab <= 0 || row_stride < vocab || n_rows < 0) return PB_E_INVALID;
  if (vocab >= PB_MAX_VOCAB) return PB_E_TOO_LARGE;
  float* x = (float*)malloc((size_t)vocab * 4);
  ent_t* ent = (ent_t*)malloc((size_t)vocab * sizeof(ent_t));
  if (!x || !ent) { free(x); free(ent); return PB_E_INVALID; }
  int rc = PB_OK;
  for (int64_t i = 0; i < n_rows; i++) {
    int64_t r = row_index ? row_index[i] : i;
    if (load_row(logits, dtype, r, vocab, row_stride, x)) { rc = PB_E_INVALID; break; }
    sample_row(x, vocab, &params[i], ent, &out_token[i], out_info ? &out_info[i] : NULL,
               out_probs ? out_probs + i * vocab : NULL);
  }
  free(x);
  free(ent);
  return rc;
}

/* kept mask of one row from its pb_row_info (for tests): 1 where the position is kept */
int pbo_kept_mask(const float* keys_or_raw, int64_t V, const pb_row_info* info, int greedy_row,
                  double temperature, uint8_t* mask) {
  const float tf = (float)temperature;
  int32_t tie_seen = 0;
  for (int64_t j = 0; j < V; j++) {
    float y = greedy_row ? keys_or_raw[j] : keys_or_raw[j] / tf;
    uint32_t k = pbo_key(y);
    uint8_t keep = 0;
    if (k > info->thr_key) keep = 1;
    else if (k == info->thr_key) { keep = tie_seen < info->n_tie_kept; tie_seen++; }
    mask[j] = keep;
  }
  return 0;
}
