/*
 * mtr_oracle.c -- CPU oracle of the fused decode-sampling step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA path is
 * compared against; it is never linked into, loaded by or called from the
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.
 *
 * It restates, row by row with plain loops and sorts, the chain the
 * reference runs after every decoder step, in the reference's processor
 * order (osuT5/osuT5/inference/logit_processors.py:240-307, then the HF
 * warpers generate() appends, transformers generation/utils.py:1212-1224):
 *
 *   CFG            out = second + (first - second) * scale, three rounded fp32
 *                  ops (transformers generation/logits_process.py:2160-2174;
 *                  "first" is the first half of the rows, HF's "cond")
 *   monotonic      ids in [ts_start, ts_start + last_value) -> -inf while the
 *                  last structural token is a time shift
 *                  (logit_processors.py:190-229; state form: optimized/single/logits.py:33-105)
 *   timeshift bias scores[:, ts_start:ts_end] += bias (logit_processors.py:35-43)
 *   grammar        allowed(v) = class transition table of the previous token
 *                  (no reference implementation; restated from the workload spec)
 *   penalties      repetition (transformers logits_process.py:407-413:
 *                  s < 0 ? s * p : s / p, once per distinct id), then
 *                  frequency s -= f * count, then presence s -= p * [count > 0]
 *                  (the last two have no reference implementation)
 *   temperature    scores / T, IEEE division with T rounded to fp32
 *                  (logits_process.py:297-301; per-row conditional form:
 *                  logit_processors.py:75-119, first match in list order)
 *   lookback       LookbackBiasLogitsWarper (logit_processors.py:122-170):
 *                  types_first = False masks [lb_start, lb_end); True
 *                  renormalises away that range after a timed-event token
 *                  (lookback_renorm below)
 *   top-k          remove scores < k-th largest score (ties kept)
 *                  (logits_process.py:581-588)
 *   top-p          nucleus over probabilities, see below
 *                  (logits_process.py:521-535 and compiled_decode.py:1147-1155)
 *   draw           inverse CDF in token-id order from a caller uniform
 *                  (replaces softmax + torch.multinomial, decode_loop.py:296-301)
 *
 * Decision arithmetic.  Probabilities are fixed point: q = floor(e^(x - max)
 * * 2^31) from mtr_oracle_expfx (Cody-Waite range reduction with ln 2 split
 * in two, then a degree-6 minimax polynomial fitted for this project on
 * [-ln2/2, ln2/2], evaluated by Horner with fused multiply-adds).  Sums of q
 * are exact 64-bit integers, so the keep set and the drawn id do not depend
 * on summation order.  Canonical order is (score descending, token id
 * ascending); top-p keeps a prefix of it:
 *     HF mode:      keep while mass_above <  top_p * Q   (TopPLogitsWarper)
 *     _sample mode: keep while mass_above <= top_p * Q   (compiled_decode._sample)
 * with P = (double)top_p * (double)Q and integer limits ceil(P) - 1 / floor(P).
 * The draw picks the smallest id whose inclusive kept-mass prefix exceeds
 * floor((double)u * (double)Q_kept).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off; no fast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/mtr_sampler.h"

/* ---- fixed-point exponential (shared definition with the CUDA kernel) ---- */
#define FX_LOG2E 0x1.715476p+0f
#define FX_LN2_HI 0x1.62e400p-1f
#define FX_LN2_LO 0x1.7f7d1cp-20f
#define FX_C0 0x1.000000p+31f
#define FX_C1 0x1.000000p+31f
#define FX_C2 0x1.fffffap+29f
#define FX_C3 0x1.55540ap+28f
#define FX_C4 0x1.55589ap+26f
#define FX_C5 0x1.126d0cp+24f
#define FX_C6 0x1.6ab980p+21f

uint32_t mtr_oracle_expfx(float d) {
  if (!(d >= -32.0f)) return 0u; /* also -inf */
  float n = rintf(d * FX_LOG2E);
  float r = fmaf(-n, FX_LN2_HI, d);
  r = fmaf(-n, FX_LN2_LO, r);
  float p = FX_C6;
  p = fmaf(p, r, FX_C5);
  p = fmaf(p, r, FX_C4);
  p = fmaf(p, r, FX_C3);
  p = fmaf(p, r, FX_C2);
  p = fmaf(p, r, FX_C1);
  p = fmaf(p, r, FX_C0);
  uint32_t m = (uint32_t)p;
  int sh = -(int)n;
  return sh >= 32 ? 0u : (m >> sh);
}

/* Markstein division with a precomputed reciprocal; exported so the CPU
 * tests can check it against IEEE division (the kernel uses it for
 * temperature, the oracle itself always divides). */
float mtr_oracle_markstein_div(float x, float t) {
  float y = 1.0f / t;
  float q0 = x * y;
  float r = fmaf(-q0, t, x);
  return fmaf(r, y, q0);
}

/* ---- element access ---- */
static float half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        e++;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static float load_logit(const MtrSamplerArgs* a, int64_t row, int64_t v) {
  int64_t off = row * a->logits_row_stride + v;
  if (a->logits_dtype == MTR_DTYPE_F32) return ((const float*)a->logits)[off];
  uint16_t h = ((const uint16_t*)a->logits)[off];
  if (a->logits_dtype == MTR_DTYPE_BF16) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
  }
  return half_to_float(h);
}

static int64_t load_id(const MtrSamplerArgs* a, int64_t row, int64_t pos) {
  int64_t off = row * a->ids_row_stride + pos;
  if (a->ids_dtype == MTR_IDS_I32) return ((const int32_t*)a->input_ids)[off];
  return ((const int64_t*)a->input_ids)[off];
}

static int is_sos(const MtrSamplerArgs* a, int64_t tok) {
  for (int i = 0; i < a->n_sos; ++i)
    if (tok == a->sos_ids[i]) return 1;
  return 0;
}

/* stateful monotonic update (optimized/single/logits.py:85-105) */
static int32_t mono_update(const MtrSamplerArgs* a, int32_t s, int64_t tok) {
  if (tok >= a->ts_start && tok < a->ts_end) return (int32_t)(tok - a->ts_start);
  if (is_sos(a, tok)) return -1;
  return s;
}

static int is_eos(const MtrSamplerArgs* a, int64_t tok) {
  for (int i = 0; i < a->n_eos; ++i)
    if (tok == a->eos_ids[i]) return 1;
  for (int i = 0; i < a->n_eos_ranges; ++i)
    if (tok >= a->eos_range_start[i] && tok < a->eos_range_end[i]) return 1;
  return 0;
}

typedef struct {
  float x;
  int32_t id;
} Ent;

static int cmp_canonical(const void* pa, const void* pb) {
  const Ent* a = (const Ent*)pa;
  const Ent* b = (const Ent*)pb;
  if (a->x > b->x) return -1;
  if (a->x < b->x) return 1;
  return (a->id > b->id) - (a->id < b->id);
}

static int cmp_float_desc(const void* pa, const void* pb) {
  float a = *(const float*)pa, b = *(const float*)pb;
  return (a < b) - (a > b);
}

static const float NEG_INF = -INFINITY;

/* ln x in double: x = f 2^e with f in [sqrt(1/2), sqrt(2)), ln x = e ln2 +
 * 2 atanh(z), z = (f - 1) / (f + 1), atanh by its odd series to z^23 (|z| <=
 * 0.172).  Each step is one IEEE double operation (no contraction), the same
 * sequence the kernel runs.  Exported for the CPU tests. */
double mtr_oracle_log_d(double x) {
  static const double C[12] = {
      1.0,
      0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3, 0x1.c71c71c71c71cp-4,
      0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4, 0x1.e1e1e1e1e1e1ep-5,
      0x1.af286bca1af28p-5, 0x1.8618618618618p-5, 0x1.642c8590b2164p-5,
  };
  if (x != x) return x;
  if (x < 0.0) return NAN;
  if (x == 0.0) return -INFINITY;
  if (x == INFINITY) return x;
  int e = 0;
  uint64_t b;
  memcpy(&b, &x, 8);
  if ((b >> 52) == 0) {
    x = x * 0x1p54;
    memcpy(&b, &x, 8);
    e = -54;
  }
  e += (int)(b >> 52) - 1023;
  b = (b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;
  double f;
  memcpy(&f, &b, 8);
  if (f > 0x1.6a09e667f3bcdp+0) {
    f = f * 0.5;
    e += 1;
  }
  double z = (f - 1.0) / (f + 1.0);
  double w = z * z;
  double p = C[11];
  for (int k = 10; k >= 0; --k) p = p * w + C[k];
  return (double)e * 0x1.62e42fefa39efp-1 + (2.0 * z) * p;
}

/* LookbackBiasLogitsWarper, types_first = True
 * (osuT5/osuT5/inference/logit_processors.py:143-170), on one row of scores
 * after temperature.  p = the previous step's EOS probability (lb_state, NaN:
 * no previous step), masses in fixed point: Q over every finite score, O over
 * the ids outside [lb_start, lb_end), E over the EOS ids (a repeated id counts
 * each time, as the reference's index-and-sum does).  When the last input id
 * is a timed-event token and p is known:
 *   s = 1 / ((O/Q)(1 - p) + p)
 *   x -> x - c, c = max + ln(Q 2^-31) - ln s        outside the range
 *   x -> -inf                                       inside the range
 *   x[lb_start] = ln(clip((s - 1) p / (1 - p), 0, 1))
 * The row's new state is E / Q of the scores BEFORE the transform (the
 * reference keeps last_scores = its input); a row with NaN or +inf scores, or
 * all -inf, stores NaN and is left as it is. */
static void lookback_renorm(const MtrSamplerArgs* a, int64_t r, int32_t L, float* xs, int32_t V) {
  float m = NEG_INF;
  int bad = 0;
  for (int32_t v = 0; v < V; ++v) {
    float x = xs[v];
    if (x != x || x == INFINITY) bad = 1;
    else if (x > m) m = x;
  }
  const float p_prev = a->lb_state[r];
  if (bad || m == NEG_INF) {
    a->lb_state[r] = NAN;
    return;
  }
  uint64_t Q = 0, O = 0, E = 0;
  for (int32_t v = 0; v < V; ++v) {
    if (!(xs[v] > NEG_INF)) continue;
    uint32_t q = mtr_oracle_expfx(xs[v] - m);
    Q += q;
    if (v < a->lb_start || v >= a->lb_end) O += q;
  }
  for (int k = 0; k < a->n_lb_eos; ++k) {
    int32_t id = a->lb_eos_ids[k];
    if (xs[id] > NEG_INF) E += mtr_oracle_expfx(xs[id] - m);
  }
  a->lb_state[r] = (float)((double)E / (double)Q);
  int timed = 0;
  if (L > 0) {
    int64_t t = load_id(a, r, L - 1);
    timed = t >= 0 && t < V && ((a->lb_timed_bits[t >> 5] >> (t & 31)) & 1u);
  }
  if (!timed || p_prev != p_prev) return;
  const double p = (double)p_prev, pe = 1.0 - p;
  const double ratio = (double)O / (double)Q;
  const double s = 1.0 / (ratio * pe + p);
  double ex = (s - 1.0) * p / pe;
  if (ex < 0.0) ex = 0.0;
  else if (ex > 1.0) ex = 1.0;
  const double lq = mtr_oracle_log_d((double)Q) - 31.0 * 0x1.62e42fefa39efp-1;
  const double c = ((double)m + lq) - mtr_oracle_log_d(s);
  for (int32_t v = 0; v < V; ++v)
    xs[v] = (v >= a->lb_start && v < a->lb_end) ? NEG_INF : (float)((double)xs[v] - c);
  xs[a->lb_start] = (float)mtr_oracle_log_d(ex);
}

/* sizeof(MtrSamplerArgs) this oracle was compiled with (layout check). */
size_t mtr_oracle_args_size(void) { return sizeof(MtrSamplerArgs); }

/* Processes every row; host pointers throughout.  Returns 0. */
int mtr_oracle_run(const MtrSamplerArgs* a) {
  const int64_t B = a->num_rows;
  const int32_t V = a->vocab;
  const int32_t L = a->input_ids ? a->ids_len : 0;
  const int64_t second = a->cfg_second_offset > 0 ? a->cfg_second_offset : B;
  const int pen_on = a->repetition_penalty != 1.0f || a->frequency_penalty != 0.0f ||
                     a->presence_penalty != 0.0f;
  float* xs = (float*)malloc(sizeof(float) * (size_t)V);
  uint32_t* q = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)V);
  uint32_t* cnt = (uint32_t*)calloc((size_t)V, sizeof(uint32_t));
  Ent* ord = (Ent*)malloc(sizeof(Ent) * (size_t)V);
  float* vals = (float*)malloc(sizeof(float) * (size_t)V);

  for (int64_t r = 0; r < B; ++r) {
    uint32_t status = 0;

    /* ---- monotonic state ---- */
    int32_t mono = -1;
    if (a->mono_mode == MTR_MONO_STATE) {
      mono = a->mono_state ? a->mono_state[r] : -1;
      if ((a->flags & MTR_FLAG_MONO_UPDATE_FROM_IDS) && L > 0)
        mono = mono_update(a, mono, load_id(a, r, L - 1));
    } else if (a->mono_mode == MTR_MONO_SCAN) {
      int64_t last_ts = -1, last_sos = -1;
      for (int64_t i = 0; i < L; ++i) {
        int64_t t = load_id(a, r, i);
        if (t >= a->ts_start && t < a->ts_end) last_ts = i;
        if (is_sos(a, t)) last_sos = i;
      }
      mono = (last_ts != -1 && last_ts > last_sos)
                 ? (int32_t)(load_id(a, r, last_ts) - a->ts_start)
                 : -1;
    }
    const int64_t mono_hi = mono >= 0 ? (int64_t)a->ts_start + mono : -1;

    /* ---- grammar ---- */
    int grammar = 0;
    uint32_t allow = 0xffffffffu;
    if (a->grammar_class_of) {
      int64_t prev = -1;
      if (a->flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS)
        prev = L > 0 ? load_id(a, r, L - 1) : -1;
      else if (a->prev_token)
        prev = a->prev_token[r];
      if (prev >= V) status |= MTR_ROW_BAD_ID;
      if (prev >= 0 && prev < V) {
        uint32_t c = a->grammar_class_of[prev];
        if (c < (uint32_t)a->grammar_n_classes) {
          grammar = 1;
          allow = a->grammar_allow[c];
        } else {
          status |= MTR_ROW_BAD_ID;
        }
      }
    }

    /* ---- per-row temperature ---- */
    float t_row = a->temperature;
    if (a->temp_mode == MTR_TEMP_ROW_CONDITIONAL) {
      for (int c = 0; c < a->n_cond; ++c) {
        int off = a->cond_offset[c];
        if (off < 1 || L < off) continue;
        int64_t tok = load_id(a, r, L - off);
        if (tok >= 0 && tok < V && ((a->cond_token_bits[c][tok >> 5] >> (tok & 31)) & 1u)) {
          t_row = a->cond_temperature[c];
          break;
        }
      }
    }

    /* ---- penalties: counts over the history ---- */
    if (pen_on) {
      memset(cnt, 0, sizeof(uint32_t) * (size_t)V);
      for (int64_t i = a->penalty_start; i < L; ++i) {
        int64_t t = load_id(a, r, i);
        if (t < 0 || t >= V) {
          status |= MTR_ROW_BAD_ID;
          continue;
        }
        cnt[t]++;
      }
    }

    /* ---- elementwise chain ---- */
    for (int32_t v = 0; v < V; ++v) {
      float x = load_logit(a, r, v);
      if (a->cfg_enabled) {
        float s = load_logit(a, r + second, v);
        float d = x - s;
        float m = d * a->cfg_scale;
        x = s + m;
      }
      if (mono_hi >= 0 && v >= a->ts_start && v < a->ts_end && v < mono_hi) x = NEG_INF;
      if (a->timeshift_bias != 0.0f && v >= a->ts_start && v < a->ts_end) x = x + a->timeshift_bias;
      if (grammar) {
        uint32_t c = a->grammar_class_of[v];
        if (!(c < (uint32_t)a->grammar_n_classes && ((allow >> c) & 1u))) x = NEG_INF;
      }
      if (pen_on && cnt[v] > 0) {
        if (a->repetition_penalty != 1.0f)
          x = x < 0.0f ? x * a->repetition_penalty : x / a->repetition_penalty;
        if (a->frequency_penalty != 0.0f) {
          float f = a->frequency_penalty * (float)cnt[v];
          x = x - f;
        }
        if (a->presence_penalty != 0.0f) x = x - a->presence_penalty;
      }
      float t = t_row;
      if (a->temp_mode == MTR_TEMP_COLUMN_RANGES) {
        for (int k = 0; k < a->n_col_ranges; ++k)
          if (v >= a->col_start[k] && v < a->col_end[k]) {
            t = a->col_temperature[k];
            break;
          }
      }
      if (t != 1.0f) x = x / t;
      xs[v] = x;
    }

    /* ---- lookback bias (logit_processors.py:143-170) ---- */
    if (a->lookback_mode == MTR_LOOKBACK_MASK) {
      for (int32_t v = a->lb_start; v < a->lb_end && v < V; ++v) xs[v] = NEG_INF;
    } else if (a->lookback_mode == MTR_LOOKBACK_RENORM) {
      lookback_renorm(a, r, L, xs, V);
    }

    /* ---- row statistics ---- */
    /* torch.argmax semantics: first NaN if any, else first maximum (index 0
     * for an all -inf row) */
    int nonfinite = 0;
    int32_t first_nan = -1;
    float mx = NEG_INF;
    int32_t amax = 0;
    int64_t nfinite = 0;
    for (int32_t v = 0; v < V; ++v) {
      float x = xs[v];
      if (isnan(x)) {
        nonfinite = 1;
        if (first_nan < 0) first_nan = v;
        continue;
      }
      if (x == INFINITY) nonfinite = 1;
      if (x > mx) {
        mx = x;
        amax = v;
      }
      if (x > NEG_INF && x < INFINITY) nfinite++;
    }
    if (first_nan >= 0) amax = first_nan;
    if (mx == NEG_INF && !nonfinite) status |= MTR_ROW_ALL_MASKED;
    if (nonfinite) status |= MTR_ROW_NONFINITE;

    int64_t token = -1;
    int clean = !(status & (MTR_ROW_NONFINITE | MTR_ROW_ALL_MASKED));
    uint64_t qkept = 0;

    if (a->select_mode == MTR_SELECT_ARGMAX) {
      token = amax;
      if (clean) {
        for (int32_t v = 0; v < V; ++v) {
          q[v] = (xs[v] > NEG_INF) ? mtr_oracle_expfx(xs[v] - mx) : 0u;
          qkept += q[v];
        }
      }
    } else if (clean) {
      /* ---- top-k ---- */
      if (a->top_k > 0 && (int64_t)a->top_k < nfinite) {
        int64_t n = 0;
        for (int32_t v = 0; v < V; ++v)
          if (xs[v] > NEG_INF) vals[n++] = xs[v];
        qsort(vals, (size_t)n, sizeof(float), cmp_float_desc);
        float tk = vals[a->top_k - 1];
        for (int32_t v = 0; v < V; ++v)
          if (xs[v] < tk) xs[v] = NEG_INF;
      }
      uint64_t qtot = 0;
      for (int32_t v = 0; v < V; ++v) {
        q[v] = (xs[v] > NEG_INF) ? mtr_oracle_expfx(xs[v] - mx) : 0u;
        qtot += q[v];
      }
      /* ---- top-p ---- */
      if (a->top_p < 1.0f) {
        double P = (double)a->top_p * (double)qtot;
        uint64_t plim = a->top_p_mode == MTR_TOPP_HF ? (uint64_t)ceil(P) - 1u : (uint64_t)floor(P);
        int64_t n = 0;
        for (int32_t v = 0; v < V; ++v)
          if (xs[v] > NEG_INF) {
            ord[n].x = xs[v];
            ord[n].id = v;
            n++;
          }
        qsort(ord, (size_t)n, sizeof(Ent), cmp_canonical);
        uint64_t above = 0;
        int64_t last = -1;
        for (int64_t i = 0; i < n; ++i) {
          int32_t id = ord[i].id;
          if (above <= plim) {
            last = i;
          } else {
            xs[id] = NEG_INF;
          }
          above += q[id];
        }
        if (last >= 0 && last + 1 < n && ord[last + 1].x == ord[last].x) status |= MTR_ROW_TIE_AT_CUT;
      }
      for (int32_t v = 0; v < V; ++v)
        if (xs[v] > NEG_INF) qkept += q[v];
      /* ---- draw ---- */
      if (a->select_mode == MTR_SELECT_SAMPLE) {
        float u = a->uniforms[r];
        if (!(u >= 0.0f)) {
          u = 0.0f;
          status |= MTR_ROW_BAD_UNIFORM;
        } else if (u >= 1.0f) {
          u = 0x1.fffffep-1f;
          status |= MTR_ROW_BAD_UNIFORM;
        }
        uint64_t target = (uint64_t)floor((double)u * (double)qkept);
        uint64_t c = 0;
        for (int32_t v = 0; v < V; ++v) {
          if (xs[v] > NEG_INF) {
            c += q[v];
            if (c > target) {
              token = v;
              break;
            }
          }
        }
      }
    } else if (a->select_mode == MTR_SELECT_SAMPLE) {
      token = a->pad_id;
    }

    /* ---- outputs ---- */
    if (a->out_scores)
      for (int32_t v = 0; v < V; ++v) a->out_scores[r * a->out_scores_row_stride + v] = xs[v];
    if (a->out_logprobs) {
      float* lp = a->out_logprobs + r * a->out_logprobs_row_stride;
      if (!clean) {
        for (int32_t v = 0; v < V; ++v) lp[v] = NAN;
      } else {
        double lse = log((double)qkept) - 31.0 * 0.69314718055994530942;
        for (int32_t v = 0; v < V; ++v)
          lp[v] = xs[v] > NEG_INF ? (float)(((double)xs[v] - (double)mx) - lse) : NEG_INF;
      }
    }
    if (a->select_mode != MTR_SELECT_NONE) {
      /* pad, EOS, append, stop counters (decode_loop.py:303-316, compiled_decode.py:1072-1080) */
      int64_t final_tok = token;
      int live = 1;
      if (a->unfinished) {
        live = a->unfinished[r] != 0;
        if (!live) final_tok = a->pad_id;
      }
      int eos = is_eos(a, final_tok);
      if (a->unfinished) a->unfinished[r] = (uint8_t)(live && !eos);
      if (a->stop_counts && live && eos) {
        a->stop_counts[0] += 1u;
        if (a->unfinished) a->stop_counts[1] += 1u;
      }
      if (a->id_buffer) {
        int32_t cur = a->cur_len_dev ? *a->cur_len_dev : a->cur_len;
        if (cur >= 0 && (int64_t)cur < a->id_buffer_row_stride)
          a->id_buffer[r * a->id_buffer_row_stride + cur] = final_tok;
        else
          status |= MTR_ROW_APPEND_SKIPPED;
      }
      if (a->flags & MTR_FLAG_MONO_UPDATE_FROM_SAMPLE) mono = mono_update(a, mono, final_tok);
      if ((a->flags & MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE) && a->prev_token)
        a->prev_token[r] = (int32_t)final_tok;
      if (a->out_ids) a->out_ids[r] = final_tok;
    }
    if (a->mono_mode != MTR_MONO_OFF && a->mono_state) a->mono_state[r] = mono;
    if (a->out_status) a->out_status[r] = status;
  }
  free(xs);
  free(q);
  free(cnt);
  free(ord);
  free(vals);
  return 0;
}

/* Counts x (every `stride`-th float with binade in [e_lo, e_hi), both signs)
 * for which the Markstein sequence differs from IEEE x / t.  CPU test aid. */
uint64_t mtr_oracle_markstein_mismatches(float t, int e_lo, int e_hi, uint32_t stride) {
  uint64_t bad = 0;
  const float y = 1.0f / t;
  for (int e = e_lo; e < e_hi; ++e) {
    for (uint32_t m = 0; m < (1u << 23); m += stride) {
      uint32_t bits = ((uint32_t)(e + 127) << 23) | m;
      for (int s = 0; s < 2; ++s) {
        uint32_t b = bits | (s ? 0x80000000u : 0u);
        float x;
        memcpy(&x, &b, 4);
        float q0 = x * y;
        float r = fmaf(-q0, t, x);
        float q = fmaf(r, y, q0);
        if (q != x / t) bad++;
      }
    }
  }
  return bad;
}
