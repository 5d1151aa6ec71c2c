/*
 * mtr_sampler.h -- C ABI of the fused decode-sampling step (logits-processor
 * chain + token sampler) for Mapperatorinator-style event-token decoders on
 * NVIDIA B200 (sm_100a).
 *
 * One call processes B output rows of a [R, V] logits matrix (R = B, or 2B
 * with classifier-free guidance) and, depending on `select_mode`, writes the
 * processed scores, the greedy token or a token drawn from caller-supplied
 * uniforms.  All buffers are caller-owned device memory; the library
 * allocates nothing, never synchronises the stream and never throws.  Every
 * entry point returns an MtrStatus code.
 *
 * Reference interfaces replaced (paths are inside the Mapperatorinator
 * project; "HF:" means transformers/generation/ of the pinned transformers):
 *   mtr_sampler_launch, select_mode = MTR_SELECT_NONE
 *       replaces LogitsProcessorList.__call__ over the chain built by
 *       build_logits_processor_list (osuT5/osuT5/inference/logit_processors.py:240-307)
 *       -- ClassifierFreeGuidanceLogitsProcessor (HF:logits_process.py:2160-2174),
 *       MonotonicTimeShiftLogitsProcessor (logit_processors.py:173-237),
 *       TimeshiftBias (logit_processors.py:35-43),
 *       ConditionalTemperatureLogitsWarper (logit_processors.py:46-119),
 *       TemperatureLogitsWarper (HF:logits_process.py:297-301) -- followed by the
 *       warpers generate() appends: TopKLogitsWarper (HF:logits_process.py:581-588)
 *       and TopPLogitsWarper (HF:logits_process.py:521-535).
 *   mtr_sampler_launch, select_mode = MTR_SELECT_ARGMAX / MTR_SELECT_SAMPLE
 *       replaces _sample(logits, do_sample, top_p, top_k, temperature)
 *       (osuT5/osuT5/inference/compiled_decode.py:1135-1158) and the
 *       softmax + torch.multinomial / argmax block of the decode loops
 *       (osuT5/osuT5/inference/optimized/single/decode_loop.py:289-301,
 *       HF:utils.py:2762-2793), plus the pad-on-finished step
 *       (decode_loop.py:303-305).
 *   mono_state (MTR_MONO_STATE) replaces the per-row state of the stateful
 *       monotonic processors (osuT5/osuT5/inference/optimized/single/logits.py:13-113,
 *       compiled_decode.py:309-372).
 */
#ifndef MTR_SAMPLER_H
#define MTR_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MTR_ABI_VERSION 2

/* Limits (also reported by mtr_sampler_query). */
#define MTR_MAX_VOCAB 131072
#define MTR_MAX_IDS_LEN 65535
#define MTR_MAX_SOS_IDS 16
#define MTR_MAX_COND_TEMPS 4
#define MTR_MAX_COL_TEMP_RANGES 8
#define MTR_MAX_GRAMMAR_CLASSES 32
#define MTR_MAX_EOS_IDS 16
#define MTR_MAX_EOS_RANGES 2
#define MTR_MAX_LB_EOS 8

/* Return codes of every entry point. */
typedef enum MtrStatus {
  MTR_OK = 0,
  MTR_ERR_NULL_ARG = 1,     /* a required pointer is NULL */
  MTR_ERR_BAD_SHAPE = 2,    /* vocab / rows / strides / ids_len out of range */
  MTR_ERR_BAD_PARAM = 3,    /* a scalar parameter out of its domain */
  MTR_ERR_UNSUPPORTED = 4,  /* a valid request this build cannot serve */
  MTR_ERR_ALIGNMENT = 5,    /* a pointer is not aligned to its element size */
  MTR_ERR_CUDA = 6,         /* the CUDA runtime reported an error */
  MTR_ERR_ABI = 7           /* abi_version / struct_size mismatch */
} MtrStatus;

/* Per-row status bits written to out_status (0 = clean row). */
#define MTR_ROW_NONFINITE   (1u << 0) /* a processed score is NaN or +inf        */
#define MTR_ROW_ALL_MASKED  (1u << 1) /* every processed score is -inf           */
#define MTR_ROW_BAD_ID      (1u << 2) /* an input id outside [0, vocab) was skipped */
#define MTR_ROW_BAD_UNIFORM (1u << 3) /* uniform outside [0, 1) was clamped      */
#define MTR_ROW_SLOW_PATH   (1u << 4) /* exact radix fallback was used (info)     */
#define MTR_ROW_TIE_AT_CUT  (1u << 5) /* the top-p cut split equal scores (info)  */
#define MTR_ROW_COPY_TIMEOUT (1u << 6) /* a staged row copy never landed: this row and every later row of
                                          the same CTA get pad_id and this bit (row-per-warp kernel) */
#define MTR_ROW_APPEND_SKIPPED (1u << 7) /* the id-buffer column (*cur_len_dev) was outside [0, row stride):
                                           the token was not appended */

typedef enum MtrDType { MTR_DTYPE_F32 = 0, MTR_DTYPE_BF16 = 1, MTR_DTYPE_F16 = 2 } MtrDType;
typedef enum MtrIdType { MTR_IDS_I64 = 0, MTR_IDS_I32 = 1 } MtrIdType;

typedef enum MtrMonoMode {
  MTR_MONO_OFF = 0,
  MTR_MONO_STATE = 1, /* mask from mono_state[row] (-1 = inactive, else last value) */
  MTR_MONO_SCAN = 2   /* recompute the state from input_ids (full scan); stores it in
                         mono_state when that pointer is set */
} MtrMonoMode;

typedef enum MtrTempMode {
  MTR_TEMP_SCALAR = 0,          /* scores / temperature                                   */
  MTR_TEMP_ROW_CONDITIONAL = 1, /* per-row temperature picked from input_ids (first match) */
  MTR_TEMP_COLUMN_RANGES = 2    /* per-vocab-range temperature, `temperature` elsewhere    */
} MtrTempMode;

typedef enum MtrTopPMode {
  MTR_TOPP_HF = 0,       /* keep token while mass ranked strictly above it <  top_p */
  MTR_TOPP_SAMPLE_FN = 1 /* keep token while mass ranked strictly above it <= top_p */
} MtrTopPMode;

typedef enum MtrLookbackMode {
  MTR_LOOKBACK_OFF = 0,
  MTR_LOOKBACK_MASK = 1,   /* ids [lb_start, lb_end) -> -inf (types_first = False) */
  MTR_LOOKBACK_RENORM = 2  /* renormalise the range away after a timed-event token (types_first = True) */
} MtrLookbackMode;

typedef enum MtrSelect {
  MTR_SELECT_NONE = 0,   /* processor only: write out_scores / out_logprobs   */
  MTR_SELECT_ARGMAX = 1, /* greedy: first index of the maximum (top-k/p unused) */
  MTR_SELECT_SAMPLE = 2  /* inverse-CDF draw from uniforms[row]                  */
} MtrSelect;

/* flags */
#define MTR_FLAG_MONO_UPDATE_FROM_IDS       (1u << 0) /* fold input_ids[:, -1] into mono_state before masking */
#define MTR_FLAG_MONO_UPDATE_FROM_SAMPLE    (1u << 1) /* fold the emitted token into mono_state after the draw */
#define MTR_FLAG_GRAMMAR_PREV_FROM_IDS      (1u << 2) /* previous token = input_ids[:, -1] instead of prev_token */
#define MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE (1u << 3) /* prev_token[row] = emitted token after the draw        */
#define MTR_FLAG_FORCE_RADIX                (1u << 4) /* test hook: always take the exact radix selection path  */
#define MTR_FLAG_KERNEL_ROW_CTA             (1u << 5) /* use the row-per-CTA kernel (default: chosen by shape)  */
#define MTR_FLAG_KERNEL_ROW_WARP            (1u << 6) /* use the row-per-warp kernel (V <= 4096, <= 32767 penalty ids) */
#define MTR_FLAG_KERNEL_STREAM              (1u << 7) /* use the streaming row-group kernel (sampling or processor
                                                         output with 1 <= top_k <= 64 < V, V % 8 == 0,
                                                         V <= 65536, 16-byte aligned rows, no column
                                                         temperatures, grammar given as vocabulary bitmaps) */
#define MTR_FLAG_TEST_COPY_TIMEOUT          (1u << 8) /* test hook: the row-per-warp kernel's first staged-copy
                                                         wait gives up at once (exercises MTR_ROW_COPY_TIMEOUT) */

/*
 * All pointer fields are device pointers (host pointers for the CPU oracle
 * that shares this struct).  Optional pointers may be NULL.  Initialise with
 * mtr_args_init() and then set what is needed.
 */
typedef struct MtrSamplerArgs {
  uint32_t abi_version; /* = MTR_ABI_VERSION */
  uint32_t struct_size; /* = sizeof(MtrSamplerArgs) */

  /* ---- logits [rows, vocab], row i and (with CFG) row i + cfg_second_offset ---- */
  const void* logits;
  int64_t logits_row_stride; /* elements */
  int64_t cfg_second_offset; /* rows; <= 0 means num_rows */
  int32_t logits_dtype;      /* MtrDType */
  int32_t num_rows;          /* B = output rows */
  int32_t vocab;             /* V */
  int32_t cfg_enabled;       /* out = second + (first - second) * cfg_scale */
  float cfg_scale;
  uint32_t flags;

  /* ---- token history input_ids [B, ids_len] (CFG: one row per output row) ---- */
  const void* input_ids;
  int64_t ids_row_stride; /* elements */
  int32_t ids_dtype;      /* MtrIdType */
  int32_t ids_len;        /* L (0 allowed) */
  int32_t penalty_start;  /* penalties use input_ids[:, penalty_start:] */

  /* ---- monotonic time-shift mask ---- */
  int32_t mono_mode; /* MtrMonoMode */
  int32_t ts_start;  /* time-shift token ids are [ts_start, ts_end) */
  int32_t ts_end;
  int32_t n_sos;
  int32_t sos_ids[MTR_MAX_SOS_IDS];
  int32_t* mono_state; /* [B] */
  float timeshift_bias; /* added to [ts_start, ts_end) when != 0 */

  /* ---- event-grammar mask: allowed(v) = bit class_of[v] of allow[class_of[prev]] ---- */
  const uint8_t* grammar_class_of; /* [V] or NULL (grammar off) */
  const uint32_t* grammar_allow;   /* [grammar_n_classes] */
  /* Optional [grammar_n_classes][ceil(V/32)] bitmaps: bit v of row c is
   * (allow[c] >> class_of[v]) & 1.  When set the kernel masks 8 ids per
   * lookup instead of one class byte per id; it must agree with
   * class_of / allow (callers build it once per grammar table). */
  const uint32_t* grammar_vocab_bits;
  int32_t grammar_n_classes;
  int32_t* prev_token; /* [B]; < 0 = no previous token (no mask) */

  /* ---- penalties (off at 1 / 0 / 0) ---- */
  float repetition_penalty;
  float frequency_penalty;
  float presence_penalty;

  /* ---- temperature ---- */
  int32_t temp_mode; /* MtrTempMode */
  float temperature; /* base / scalar temperature (> 0) */
  int32_t n_cond;
  float cond_temperature[MTR_MAX_COND_TEMPS];
  int32_t cond_offset[MTR_MAX_COND_TEMPS];              /* look at input_ids[row, L - offset] */
  const uint32_t* cond_token_bits[MTR_MAX_COND_TEMPS];  /* [ceil(V/32)] membership bitmaps */
  int32_t n_col_ranges;
  int32_t col_start[MTR_MAX_COL_TEMP_RANGES];
  int32_t col_end[MTR_MAX_COL_TEMP_RANGES];
  float col_temperature[MTR_MAX_COL_TEMP_RANGES];

  /* ---- selection ---- */
  int32_t select_mode; /* MtrSelect */
  int32_t top_k;       /* 0 = off */
  float top_p;         /* 1 = off, else (0, 1) */
  int32_t top_p_mode;  /* MtrTopPMode */
  const float* uniforms; /* [B] in [0, 1); required for MTR_SELECT_SAMPLE */

  /* ---- outputs ---- */
  int64_t* out_ids; /* [B] */
  float* out_scores; /* [B, V] processed scores (filtered = -inf) */
  int64_t out_scores_row_stride;
  float* out_logprobs; /* [B, V] log-softmax of the processed scores */
  int64_t out_logprobs_row_stride;
  uint32_t* out_status; /* [B] MTR_ROW_* bits */

  /* ---- finished rows: token = unfinished ? drawn : pad_id; then unfinished &= !eos ---- */
  uint8_t* unfinished; /* [B] or NULL */
  int64_t pad_id;      /* also the token written for rows that cannot be sampled */
  int32_t n_eos;
  int32_t eos_ids[MTR_MAX_EOS_IDS];
  int32_t n_eos_ranges;
  int32_t eos_range_start[MTR_MAX_EOS_RANGES];
  int32_t eos_range_end[MTR_MAX_EOS_RANGES];

  /* ---- lookback bias, applied after temperature (LookbackBiasLogitsWarper,
   *      osuT5/osuT5/inference/logit_processors.py:122-170).  RENORM: with p the
   *      previous step's EOS probability (lb_state[row]), P = softmax of the
   *      scores, O = P outside [lb_start, lb_end), s = 1 / (O (1 - p) + p):
   *      when the last input id is a timed-event token and p is not NaN, the
   *      scores become log(P s) outside the range, log(clip((s - 1) p / (1 - p),
   *      0, 1)) at lb_start and -inf on the rest of the range; every row's
   *      lb_state becomes this step's EOS probability (sum of P over
   *      lb_eos_ids, before the bias; NaN for a row with NaN / +inf scores or
   *      none finite).  Only the row-per-CTA kernel serves lookback. ---- */
  int32_t lookback_mode;           /* MtrLookbackMode */
  int32_t lb_start;                /* lookback time-shift ids are [lb_start, lb_end) */
  int32_t lb_end;
  int32_t n_lb_eos;
  int32_t lb_eos_ids[MTR_MAX_LB_EOS];  /* eos and context-eos ids (a repeated id counts twice) */
  const uint32_t* lb_timed_bits;   /* [ceil(V/32)] membership bitmap of timed-event ids */
  float* lb_state;                 /* [B] previous step's EOS probability, NaN = no previous step; rewritten */

  /* ---- token append and stopping (optimized/single/decode_loop.py:303-316,
   *      compiled_decode.py:1072-1080): with a selection, the emitted token
   *      (pad_id for finished rows) is also written to id_buffer[row, cur],
   *      cur = *cur_len_dev when given (a device value a CUDA graph can
   *      advance between replays), else cur_len.  stop_counts accumulates over
   *      launches (the caller zeroes it when a window starts):
   *        [0] += rows still unfinished before this step whose token is an EOS
   *               id (the compiled loop stops once it grows),
   *        [1] += rows that finished in this step (needs unfinished; the HF
   *               loop stops when it reaches B). ---- */
  int64_t* id_buffer;              /* [B, id_buffer_row_stride] int64 or NULL */
  int64_t id_buffer_row_stride;
  const int32_t* cur_len_dev;      /* device column index or NULL */
  int32_t cur_len;                 /* column index when cur_len_dev is NULL */
  int32_t reserved1;
  uint32_t* stop_counts;           /* [2] or NULL */
} MtrSamplerArgs;

/* Launch geometry chosen for a problem size (diagnostics and tests). */
typedef struct MtrLaunchInfo {
  int32_t threads;        /* threads per CTA */
  int32_t elems_per_thread;
  int32_t cluster_size;   /* CTAs per row */
  int32_t grid;           /* CTAs */
  int32_t dyn_smem_bytes; /* dynamic shared memory per CTA */
  int32_t max_vocab;      /* MTR_MAX_VOCAB */
  int32_t max_ids_len;    /* MTR_MAX_IDS_LEN */
  int32_t candidate_cap;  /* size of the exact in-bin candidate list */
  int32_t kernel;         /* 0: row-per-CTA (cluster) kernel, 1: row-per-warp kernel, 2: streaming row-group kernel */
} MtrLaunchInfo;

/*
 * The decoder's output projection on the tensor cores (tcgen05, TMA), writing
 * the bf16 logits the sampler reads:
 *   logits[r, v] = RN_bf16(sum_k hidden[r, k] * weight[v, k]), fp32 accumulation.
 * Replaces VarWhisperForConditionalGeneration.proj_out (nn.Linear(d_model,
 * vocab, bias=False) in bf16) at
 * osuT5/osuT5/model/custom_transformers/modeling_varwhisper.py:1583, 1647-1649.
 */
typedef struct MtrLmHeadArgs {
  uint32_t abi_version;         /* = MTR_ABI_VERSION */
  uint32_t struct_size;         /* = sizeof(MtrLmHeadArgs) */
  const void* hidden;           /* [rows, d_model] bf16, 16-byte aligned */
  int64_t hidden_row_stride;    /* elements, multiple of 8 */
  const void* weight;           /* [vocab, d_model] bf16 (nn.Linear weight), 16-byte aligned */
  int64_t weight_row_stride;    /* elements, multiple of 8 */
  void* logits;                 /* [rows, vocab] bf16 output, 16-byte aligned */
  int64_t logits_row_stride;    /* elements, multiple of 8 */
  int32_t rows;
  int32_t d_model;              /* multiple of 64 */
  int32_t vocab;                /* multiple of 8, <= MTR_MAX_VOCAB */
  int32_t tile_n;               /* vocabulary ids per CTA: 0 = choose, 64 or 128 */
  uint32_t* error_word;         /* device word or NULL: bits set when a bounded wait gave up */
} MtrLmHeadArgs;

/* Host-side checks of MtrLmHeadArgs (no CUDA call). */
int mtr_lmhead_validate(const MtrLmHeadArgs* args);

/* The projection alone, on `stream`. */
int mtr_lmhead_launch(const MtrLmHeadArgs* args, void* stream);

/* The projection, then mtr_sampler_launch on its logits as a programmatic
 * dependent launch (the sampler's CTAs start while the projection drains and
 * wait for its results).  sampler->logits must be lm->logits (bf16, same row
 * stride and vocabulary) and the sampler's rows must lie inside lm->rows. */
int mtr_lmhead_sample_launch(const MtrLmHeadArgs* lm, const MtrSamplerArgs* sampler, void* stream);

/* ABI identity: MTR_ABI_VERSION and sizeof(MtrSamplerArgs) of the library. */
int mtr_abi_version(void);
size_t mtr_args_size(void);

/* Fill *args with defaults: everything off, temperature 1, top_p 1, pad 0. */
int mtr_args_init(MtrSamplerArgs* args);

/* Host-side argument checks only (no CUDA call). */
int mtr_sampler_validate(const MtrSamplerArgs* args);

/* Row-per-CTA geometry for (vocab, num_rows, penalties on/off). */
int mtr_sampler_query(int32_t vocab, int32_t num_rows, int32_t with_penalties, MtrLaunchInfo* out);

/* Kernel and geometry mtr_sampler_launch would use for these exact arguments
 * (validates them first).  Without a kernel flag the streaming row-group
 * kernel is chosen whenever it serves the request (see MTR_FLAG_KERNEL_STREAM);
 * otherwise the row-per-warp kernel for more rows than one round of
 * row-per-CTA CTAs holds (3 per SM) of a vocabulary <= 4096 whose selection
 * is argmax or a top-k <= 128, else the row-per-CTA kernel.  A kernel flag the
 * request does not fit returns MTR_ERR_UNSUPPORTED. */
int mtr_sampler_query_args(const MtrSamplerArgs* args, MtrLaunchInfo* out);

/*
 * Validate and enqueue the fused step on `stream` (a cudaStream_t; NULL = the
 * legacy default stream).  The current CUDA device must own every pointer.
 * Returns MTR_OK once the kernel is enqueued.  Capturable in a CUDA graph.
 * The kernel is a programmatic dependent launch: its CTAs may be scheduled
 * while the previous kernel on the stream runs, and wait at entry until that
 * kernel has completed with its memory visible (stream order is unchanged;
 * only launch latency overlaps).
 */
int mtr_sampler_launch(const MtrSamplerArgs* args, void* stream);

/* Human-readable name of an MtrStatus code. */
const char* mtr_status_string(int code);

/* Last cudaError_t seen by mtr_sampler_launch on this thread (0 = none). */
int mtr_last_cuda_error(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MTR_SAMPLER_H */
