/*
 * pagedbatch_b200 — C ABI of the B200 (sm_100a) batched token sampler.
 *
 * This library replaces the per-row sampling call of pagedbatch:
 *   pagedbatch/sampling.py:10   sample_token(logits[V], params, generator) -> int
 * which the engine calls once per scheduled row:
 *   pagedbatch/engine.py:133-139 (LLMEngine._postprocess)
 * with one launch over a whole batch of rows [n_rows, vocab]. The per-request knobs are those of
 *   pagedbatch/config.py:134-158 (SamplingParams: temperature, top_p, top_k; greedy <=> temperature == 0).
 *
 * Plain C types only: device pointers, sizes and a cudaStream_t passed as void*. Every entry
 * point returns 0 on success or a negative PB_E* code; none aborts, none synchronises the
 * stream, none allocates device memory.
 *
 * Sampling semantics (exact, integer where it can be):
 *   key_j  = fp32(logit_j) / fp32(temperature)          IEEE fp32 division   (sampling.py:14)
 *   order  = keys descending, ties by index ascending
 *   top-k  (0 < k < vocab): keep every key >= the k-th largest key (ties kept)  (sampling.py:15-17)
 *   w_j    = pb_exp(fp32(key_j - max_key)), q_j = floor(w_j * 2^40)   (fixed-point weights)
 *   top-p  (top_p < 1): keep position j iff sum_{i<j} q_i <= floor(fp32(top_p) * sum_K q)  (sampling.py:18-25)
 *   draw   : t = floor(U53 * sum_S q / 2^53), U53 = uniform * 2^53; token = first position in
 *            `order` (restricted to the kept set S) whose inclusive prefix of q exceeds t.
 *            This is an inverse-CDF draw; the reference draws with torch.multinomial (sampling.py:26-27).
 *   greedy : argmax of the raw logits, lowest index on ties                     (sampling.py:12-13)
 */
#ifndef PAGEDBATCH_B200_H
#define PAGEDBATCH_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PB_API __attribute__((visibility("default")))
#else
#define PB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtypes of the logits buffer ------------------------------------------------------- */
#define PB_DTYPE_F32 0
#define PB_DTYPE_BF16 1
#define PB_DTYPE_F16 2

/* ---- return codes ---------------------------------------------------------------------- */
#define PB_OK 0
#define PB_E_INVALID (-1)    /* bad argument: null pointer, size, dtype, stride, alignment */
#define PB_E_TOO_LARGE (-2)  /* vocab >= PB_MAX_VOCAB */
#define PB_E_LAUNCH (-3)     /* the CUDA launch failed (cudaGetLastError after the launch) */
#define PB_E_DEVICE (-4)     /* no usable sm_100 device / attribute query failed */
#define PB_E_SCRATCH (-5)    /* pb_sample_noalloc: the batch needs more than its fixed scratch */

/* Largest vocabulary: sums of 2^40-scaled weights must fit in 64 bits. */
#define PB_MAX_VOCAB (1 << 24)

/* ---- per-row status (pb_row_info.status; the row's token is then -1) -------------------- */
#define PB_ROW_OK 0
#define PB_ROW_NONFINITE 1   /* max key is +inf/NaN or every key is -inf: the reference's
                                torch.multinomial raises on such rows (sampling.py:27) */
#define PB_ROW_BAD_UNIFORM 2 /* uniform outside [0, 1) */
#define PB_ROW_TIMEOUT 4     /* a bounded wait on a bulk copy gave up; outputs are not valid */
#define PB_ROW_INTERNAL 8    /* a selection found no element for its target (an internal error) */
#define PB_ROW_BAD_PARAMS 16 /* temperature < 0 or NaN, top_p outside (0, 1], or top_k < 0
                                (values SamplingParams rejects, config.py:146-155) */
#define PB_ROW_FALLBACK 32   /* pb_merge only: the shards' candidates cannot settle this row
                                (top-k off or above the record, or a tie group overflowing it);
                                sample it from its full row with pb_sample */

/* pb_row_info.flags: which path resolved the row (diagnostic) */
#define PB_PATH_GREEDY 1
#define PB_PATH_SMALL 2      /* top-k candidates resolved in shared memory */
#define PB_PATH_LARGE 4      /* cluster-cooperative histogram selection over the row */
#define PB_PATH_STREAM 8     /* settled by the persistent streaming kernel (with GREEDY or SMALL) */

/* One row's sampling parameters (SamplingParams, config.py:134-158, plus the row's draw). */
typedef struct pb_row_params {
  double temperature; /* 0 => greedy (config.py:156-158); else the row is divided by fp32(temperature) */
  double top_p;       /* (0, 1]; active iff top_p < 1.0 (sampling.py:18) */
  double uniform;     /* rng == 0: the [0, 1) draw for the inverse CDF (ignored for greedy rows);
                         rng & PB_RNG_PHILOX: the bits of this field are the row's 64-bit seed */
  int32_t top_k;      /* active iff 0 < top_k < vocab (sampling.py:15) */
  uint32_t rng;       /* 0: `uniform` is the draw (drawn on the host, e.g. from the request's
                         torch.Generator). PB_RNG_PHILOX | step (step < 2^31): the draw is made on
                         the device, U53 = pb_philox_u53(seed, step), so a request's draws need no
                         host work and depend only on its seed and its step */
} pb_row_params;

#define PB_RNG_PHILOX 0x80000000u

/* The device draw of a PB_RNG_PHILOX row, as an integer U53 in [0, 2^53) (the draw is U53 / 2^53):
 * Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3",
 * SC 2011) with key (seed low 32 bits, seed high 32 bits) and counter (step, 0, 0, 0); U53 is
 * (out[0] >> 11) << 32 | out[1]. Host copy of the device function. No counterpart in the
 * reference, whose draws come from torch.multinomial on the request's generator (sampling.py:27). */
PB_API uint64_t pb_philox_u53(uint64_t seed, uint32_t step);

/* Philox4x32-10 itself (host copy): ctr[4] and key[2] in, out[4] out. */
PB_API void pb_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);

/* What the sampler decided for one row (optional output; used by the parity tests). */
typedef struct pb_row_info {
  uint32_t thr_key;   /* order-preserving key of the last kept position */
  int32_t n_tie_kept; /* kept elements whose key equals thr_key (lowest indices first) */
  int32_t kept_count; /* number of kept positions */
  int32_t status;     /* PB_ROW_* */
  float max_key;      /* largest scaled key (raw logit for greedy rows) */
  int32_t flags;      /* PB_PATH_* */
  uint64_t z_q;       /* sum of q over the top-k survivors K */
  uint64_t kept_q;    /* sum of q over the kept set S */
} pb_row_info;

/*
 * Sample one token for each of n_rows rows, in one or two launches on `stream` (see
 * pb_sample_launches).
 *
 * Replaces: pagedbatch/sampling.py:10-27 sample_token, called per row at pagedbatch/engine.py:139.
 *
 *   logits      device, dtype `dtype`, row r at logits + r*row_stride elements, last dim contiguous.
 *   row_index   optional device int32[n_rows]: work item i samples logits row row_index[i]
 *               (lets the engine skip rows whose samples_token is False, engine.py:136-137).
 *   params      device pb_row_params[n_rows].
 *   out_token   device int64[n_rows]; -1 for a row whose status is not PB_ROW_OK.
 *   out_info    optional device pb_row_info[n_rows].
 *   out_probs   optional device float[n_rows * vocab]: the renormalised probabilities of the
 *               final distribution (sampling.py:26), zero outside the kept set.
 *   stream      cudaStream_t.
 */
PB_API int pb_sample(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                     const int32_t* row_index, const pb_row_params* params, int64_t* out_token,
                     pb_row_info* out_info, float* out_probs, void* stream);

/*
 * The same sampler as stream-ordered launches over a caller-provided workspace. Results are
 * identical to pb_sample. Replaces the same call as pb_sample (pagedbatch/sampling.py:10-27).
 * When every row starts on a 16-byte boundary (logits and row_stride * element size multiples of
 * 16), three launches:
 *   1. a streaming pass that reads the batch once and writes, per row, the key of the largest value
 *      of each 128-byte group (1/32 of the logits' bytes, in the workspace);
 *   2. one CTA per row that settles greedy rows and rows with 0 < top_k <= 128 from the groups that
 *      can hold their survivors (re-reading only those);
 *   3. pb_sample's cluster kernel over the other rows and the ones pass 2 could not settle.
 * Otherwise (or with the environment variable PB_WS=balanced), two launches: the persistent
 * streaming kernel in balanced mode (the batch cut into equal shares of 16-byte vectors, one per
 * SM, so a row may be split between neighbouring CTAs; each piece of a split row publishes a record
 * in the workspace and the piece that arrives last, counted on a per-row counter in the workspace,
 * merges the row), then the cluster kernel over the rows it does not take or could not settle.
 * With out_probs it runs pb_sample itself. workspace: device memory of at least
 * pb_sample_ws_bytes(n_rows, vocab, dtype) bytes (enough for either launch), 256-byte aligned, of
 * any content (every group key and record is written before it is read; the counters carry a check
 * word), not used by another call while this one runs. pb_sample_ws_launches gives the number of
 * launches for a batch (a diagnostic for benchmarks; no counterpart in the reference).
 */
PB_API int64_t pb_sample_ws_bytes(int64_t n_rows, int64_t vocab, int dtype);
PB_API int pb_sample_ws(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                        const int32_t* row_index, const pb_row_params* params, int64_t* out_token,
                        pb_row_info* out_info, float* out_probs, void* workspace, int64_t ws_bytes, void* stream);
PB_API int pb_sample_ws_launches(const void* logits, int64_t n_rows, int64_t vocab, int64_t row_stride, int dtype);

/*
 * pb_sample_ws for callers that cannot allocate device memory: no counterpart in the reference.
 * Some callers own no allocator (a plugin inside an application that manages every byte of the
 * GPU itself, or plain C code without cudaMalloc); this entry point allocates nothing and uses a
 * fixed scratch array compiled into the library instead of a workspace. Every GPU that loads the
 * library holds that array (pb_sample_noalloc_max_bytes(), 32 MiB) until the process exits.
 * Same arguments and results as pb_sample_ws without out_probs (probabilities need pb_sample).
 * It takes the three-launch form of pb_sample_ws while its group keys fit the array (up to 2092
 * rows of 128256 fp32 logits, 4185 of bf16) and the balanced form beyond; a batch too large for
 * both returns PB_E_SCRATCH and launches nothing. The first call on
 * each device looks up the array's device address; make that call before any stream capture. All
 * calls share the one array, so calls that overlap on the GPU (two streams, or two host threads)
 * race and corrupt each other's results; keep them ordered.
 */
PB_API int64_t pb_sample_noalloc_max_bytes(void);
PB_API int pb_sample_noalloc(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                             const int32_t* row_index, const pb_row_params* params, int64_t* out_token,
                             pb_row_info* out_info, void* stream);

/*
 * Vocabulary-parallel sampling (rows split by columns over N shards, as the output of a
 * tensor-parallel LM head). No counterpart in the reference, which samples whole rows; the result
 * is the same as pb_sample on the full rows: the union of every shard's top-k survivors (all
 * values >= the shard's k-th, ties kept) contains the row's top-k set and its max.
 *
 *   1. pb_candidates on every shard writes one fixed-size record per row;
 *   2. the caller all-gathers the records of the N shards (records[s][row], s = shard order);
 *   3. pb_merge on any shard turns the N records of each row into its token and pb_row_info.
 * Rows the records cannot settle come back with status PB_ROW_FALLBACK.
 */

/* Header of one row's record; `count` uint64 entries follow (key << 32 | (0xFFFFFFFF - index)). */
typedef struct pb_cand_header {
  int32_t count;   /* entries that follow */
  int32_t flags;   /* PB_ROW_* status of the shard's row (low byte) | PB_CAND_* */
  float max_key;   /* shard's largest scaled key (raw logit for greedy rows) */
  int32_t reserved;
} pb_cand_header;
#define PB_CAND_FALLBACK 0x100 /* this shard cannot describe its part of the row */
#define PB_CAND_GREEDY 0x200   /* one entry: the shard's first maximum (raw key) */
#define PB_CAND_MAX_CAP 2048   /* largest entries per record */

/* Bytes of one row's record for `cap` entries (16 + 8 * cap). */
PB_API int64_t pb_record_bytes(int32_t cap);

/*
 * Local half of a vocabulary-parallel step on one shard: columns [vocab_offset, vocab_offset +
 * shard_vocab) of every row. Arguments as pb_sample; `params` are the rows' full parameters (the
 * top_k of the whole row); out_records holds n_rows records of pb_record_bytes(cap) bytes.
 */
PB_API int pb_candidates(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab, int64_t row_stride,
                         const int32_t* row_index, const pb_row_params* params, int64_t vocab_offset, int32_t cap,
                         void* out_records, void* stream);

/*
 * pb_candidates over a caller workspace: the same records (no counterpart in the reference). For
 * shards whose rows start on 16-byte boundaries it runs the two-pass launch of pb_sample_ws in shard
 * mode (a streaming pass over the shard's group keys, then one CTA per row writing the row's
 * record, the cluster kernel for the rows it leaves); otherwise, or with a workspace smaller than
 * pb_candidates_ws_bytes(n_rows, shard_vocab, dtype), pb_candidates' own launches. workspace:
 * 256-byte aligned device memory of any content, not used by another call while this one runs.
 */
PB_API int64_t pb_candidates_ws_bytes(int64_t n_rows, int64_t shard_vocab, int dtype);
PB_API int pb_candidates_ws(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab, int64_t row_stride,
                            const int32_t* row_index, const pb_row_params* params, int64_t vocab_offset,
                            int32_t cap, void* out_records, void* workspace, int64_t ws_bytes, void* stream);

/*
 * Merge: records laid out [n_shards][n_rows][pb_record_bytes(cap)], shards in column order.
 * Writes out_token (-1 unless PB_ROW_OK) and optional out_info exactly as pb_sample would for the
 * full rows, except PB_ROW_FALLBACK rows.
 */
PB_API int pb_merge(const void* records, int32_t n_shards, int64_t n_rows, int32_t cap, const pb_row_params* params,
                    int64_t* out_token, pb_row_info* out_info, void* stream);

/*
 * Kernel launches pb_sample / pb_candidates make for a batch of this shape on the current device:
 * 1 (the cluster kernel alone) or 2 (the persistent streaming kernel over the greedy and
 * top_k <= 128 rows, then the cluster kernel over the others and the rows it could not settle).
 * No counterpart in the reference; a diagnostic for benchmarks and tests. -1 on bad arguments.
 */
PB_API int pb_sample_launches(int64_t n_rows, int64_t vocab, int dtype, int with_probs);

/*
 * Finish reasons of the rows just sampled, on the device, right after the sampler on the same
 * stream (so the engine reads tokens and reasons back together). Replaces the per-row host check
 * pagedbatch/engine.py:173-182 (LLMEngine._finish_reason), evaluated after the token is appended:
 *   stop   (1): !ignore_eos and (token == eos_id (eos_id >= 0) or token is one of the row's stop ids)
 *   length (2): otherwise, output length >= max_tokens, or total length >= max_model_len
 *   none   (0): otherwise (and for rows whose token is negative: the sampler failed them).
 *   tokens      device int64[n_rows] (the sampler's out_token)
 *   row_state   device int32[n_rows][4]: ignore_eos (0/1), output length after the token,
 *               max_tokens, prompt + output length after the token
 *   stop_offsets, stop_ids  device CSR of the rows' stop ids: row r's are
 *               stop_ids[stop_offsets[r] .. stop_offsets[r + 1]); stop_offsets has n_rows + 1 entries
 *   out_reason  device int8[n_rows]
 */
#define PB_FINISH_NONE 0
#define PB_FINISH_STOP 1
#define PB_FINISH_LENGTH 2
PB_API int pb_stop_check(const int64_t* tokens, int64_t n_rows, const int32_t* row_state, const int32_t* stop_offsets,
                         const int32_t* stop_ids, int32_t eos_id, int32_t max_model_len, int8_t* out_reason,
                         void* stream);

/* Order-preserving 32-bit key of a float (NaN above +inf, -0 == +0); host helper for tests. */
PB_API uint32_t pb_key_of(float x);

/* The fixed exp of the weights, w = pb_exp(d) for d <= 0 (host copy of the device function). */
PB_API float pb_exp(float d);

/* Short text for a PB_E* code. */
PB_API const char* pb_strerror(int code);

/* Version of this library, as major*10000 + minor*100 + patch. */
PB_API int pb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDBATCH_B200_H */
