// mtr_sampler.cu -- fused decode-sampling step for sm_100a (B200).
//
// One output row of the [B, V] processed logits is owned by one CTA, or by a
// thread-block cluster of CS CTAs when V is large.  The row lives in registers
// (THREADS x EPT elements per CTA) from the first 128-bit load to the last
// store; no intermediate B x V tensor ever reaches HBM.  Per row:
//
//   prologue   monotonic state (stateful, or a full scan of input_ids), grammar
//              row of the previous token, per-row temperature, uniform
//   load       ld.global.cs 16-byte vectors of bf16 / f16 / f32 logits; with
//              CFG the first-half row and its second-half partner
//   chain      CFG -> monotonic mask -> timeshift bias -> grammar mask ->
//              penalties (history side, shared-memory histogram) ->
//              temperature (Markstein division, bit-exact to IEEE x / T)
//   stats      max, first arg-max (NaN first, as torch.argmax), finite count
//   top-k      count histogram over d = max - x in 1/8 bins, exact k-th value
//              inside the crossing bin (candidate list, or radix fallback)
//   top-p      same scheme weighted by fixed-point probabilities
//              q = floor(e^(x - max) * 2^31); integer sums, so the keep set is
//              independent of thread order; ties at the cut go to the lowest id
//   draw       smallest id whose kept-mass prefix exceeds floor(u * Q_kept)
//   epilogue   ids, processed scores / log-probs, row status, state updates
//
// Reference arithmetic followed (paths inside the Mapperatorinator project,
// "HF:" = transformers/generation/):
//   CFG        HF:logits_process.py:2160-2174 (first half = "cond")
//   monotonic  osuT5/osuT5/inference/logit_processors.py:190-229,
//              osuT5/osuT5/inference/optimized/single/logits.py:33-105
//   bias       logit_processors.py:35-43
//   temp       HF:logits_process.py:297-301, logit_processors.py:75-119
//   top-k/p    HF:logits_process.py:521-535, 581-588;
//              osuT5/osuT5/inference/compiled_decode.py:1135-1158
//   draw       osuT5/osuT5/inference/optimized/single/decode_loop.py:296-305
//
// The kernel holds no spin-waits: every barrier is __syncthreads() or a
// hardware cluster barrier that all CTAs of the cluster reach on the same,
// row-uniform control path.
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/mtr_sampler.h"

namespace cg = cooperative_groups;

namespace mtr {

constexpr int NB = 256;             // distance bins per histogram
constexpr int CAP = 256;            // exact candidate list capacity
constexpr float BIN_SCALE = 8.0f;   // bins per logit unit
constexpr int32_t NO_ID = 0x7fffffff;

typedef unsigned long long u64;

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
__device__ __forceinline__ float pos_inf() { return __int_as_float(0x7f800000); }

// ---------------------------------------------------------------------------
// numerics
// ---------------------------------------------------------------------------

// floor(e^d * 2^31) for d <= 0, by Cody-Waite reduction (ln 2 split into a
// 16-bit head and a tail) and a degree-6 minimax polynomial on [-ln2/2, ln2/2]
// with coefficients pre-scaled by 2^31; every step is a single IEEE-rounded
// operation so the CPU oracle reproduces it bit for bit.
__device__ __forceinline__ uint32_t expfx(float d) {
  if (!(d >= -32.0f)) return 0u;
  const float n = rintf(__fmul_rn(d, 0x1.715476p+0f));
  float r = __fmaf_rn(-n, 0x1.62e400p-1f, d);
  r = __fmaf_rn(-n, 0x1.7f7d1cp-20f, r);
  float p = 0x1.6ab980p+21f;
  p = __fmaf_rn(p, r, 0x1.126d0cp+24f);
  p = __fmaf_rn(p, r, 0x1.55589ap+26f);
  p = __fmaf_rn(p, r, 0x1.55540ap+28f);
  p = __fmaf_rn(p, r, 0x1.fffffap+29f);
  p = __fmaf_rn(p, r, 0x1.000000p+31f);
  p = __fmaf_rn(p, r, 0x1.000000p+31f);
  const uint32_t m = __float2uint_rz(p);
  const int sh = -__float2int_rz(n);
  return sh >= 32 ? 0u : (m >> sh);
}

// x / t correctly rounded, given y = RN(1/t) (Markstein: q0 = x*y, r = x - q0*t
// exactly, q = q0 + r*y).  Magnitudes outside [2^-60, 2^60) and NaN take the
// IEEE divide; zeros and infinities pass through (t is positive and finite).
__device__ __forceinline__ float div_by(float x, float t, float y) {
  const float ax = fabsf(x);
  if (ax >= 0x1p-60f && ax < 0x1p60f) {
    const float q0 = __fmul_rn(x, y);
    const float r = __fmaf_rn(-q0, t, x);
    return __fmaf_rn(r, y, q0);
  }
  if (x == 0.0f || ax == pos_inf()) return x;
  return __fdiv_rn(x, t);
}

// order-preserving key of a non-NaN float (-0 and +0 share a key)
__device__ __forceinline__ uint32_t fkey(float x) {
  uint32_t u = __float_as_uint(x);
  if (x == 0.0f) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// distance bin of a finite x below the row maximum mx (monotone in x)
__device__ __forceinline__ int dbin(float mx, float x) {
  float s = __fmul_rn(__fsub_rn(mx, x), BIN_SCALE);
  s = fminf(s, (float)(NB - 1));
  return __float2int_rz(s);
}

__device__ __forceinline__ bool finite_val(float x) { return fabsf(x) < pos_inf(); }

// ---------------------------------------------------------------------------
// element loads
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int VEC = 4;
  __device__ static float get(const uint4& w, int e) {
    const uint32_t v = e == 0 ? w.x : e == 1 ? w.y : e == 2 ? w.z : w.w;
    return __uint_as_float(v);
  }
  __device__ static float one(const void* p, int64_t i) { return __ldcs((const float*)p + i); }
  static constexpr int DT = MTR_DTYPE_F32;
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int VEC = 8;
  __device__ static float get(const uint4& w, int e) {
    const uint32_t v = (e >> 1) == 0 ? w.x : (e >> 1) == 1 ? w.y : (e >> 1) == 2 ? w.z : w.w;
    return __uint_as_float((e & 1) ? (v & 0xffff0000u) : (v << 16));
  }
  __device__ static float one(const void* p, int64_t i) {
    const unsigned short h = __ldcs((const unsigned short*)p + i);
    return __uint_as_float((uint32_t)h << 16);
  }
  static constexpr int DT = MTR_DTYPE_BF16;
};
template <> struct Elem<__half> {
  static constexpr int VEC = 8;
  __device__ static float get(const uint4& w, int e) {
    const uint32_t v = (e >> 1) == 0 ? w.x : (e >> 1) == 1 ? w.y : (e >> 1) == 2 ? w.z : w.w;
    const unsigned short h = (e & 1) ? (unsigned short)(v >> 16) : (unsigned short)(v & 0xffffu);
    return __half2float(__ushort_as_half(h));
  }
  __device__ static float one(const void* p, int64_t i) {
    const unsigned short h = __ldcs((const unsigned short*)p + i);
    return __half2float(__ushort_as_half(h));
  }
  static constexpr int DT = MTR_DTYPE_F16;
};

__device__ __forceinline__ int64_t load_id(const MtrSamplerArgs& a, int64_t row, int64_t pos) {
  const int64_t off = row * a.ids_row_stride + pos;
  if (a.ids_dtype == MTR_IDS_I32) return (int64_t)__ldg((const int32_t*)a.input_ids + off);
  return (int64_t)__ldg((const long long*)a.input_ids + off);
}

__device__ __forceinline__ bool is_sos(const MtrSamplerArgs& a, int64_t t) {
  bool s = false;
#pragma unroll 1
  for (int i = 0; i < a.n_sos; ++i) s |= (t == (int64_t)a.sos_ids[i]);
  return s;
}

__device__ __forceinline__ int32_t mono_update(const MtrSamplerArgs& a, int32_t s, int64_t t) {
  if (t >= a.ts_start && t < a.ts_end) return (int32_t)(t - a.ts_start);
  if (is_sos(a, t)) return -1;
  return s;
}

__device__ __forceinline__ bool is_eos(const MtrSamplerArgs& a, int64_t t) {
  bool e = false;
#pragma unroll 1
  for (int i = 0; i < a.n_eos; ++i) e |= (t == (int64_t)a.eos_ids[i]);
#pragma unroll 1
  for (int i = 0; i < a.n_eos_ranges; ++i) e |= (t >= a.eos_range_start[i] && t < a.eos_range_end[i]);
  return e;
}

// ---------------------------------------------------------------------------
// cluster helper: CS == 1 degenerates to the CTA
// ---------------------------------------------------------------------------
template <int CS> struct Clu {
  __device__ static int rank() {
    if constexpr (CS == 1) return 0;
    else return (int)cg::this_cluster().block_rank();
  }
  __device__ static void sync() {
    if constexpr (CS == 1) __syncthreads();
    else cg::this_cluster().sync();
  }
  template <typename T> __device__ static T* at(T* p, int r) {
    if constexpr (CS == 1) return p;
    else return cg::this_cluster().map_shared_rank(p, (unsigned)r);
  }
};

// ---------------------------------------------------------------------------
// warp / block reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ u64 warp_sum_u64(u64 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ u64 warp_incl_scan_u64(u64 v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const u64 t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

struct Cross {
  int32_t bin;   // first bin whose inclusive prefix exceeds the limit (-1: none)
  int32_t pad;
  u64 above;     // weight of the bins before it
  u64 w;         // weight of that bin
  u64 total;     // weight of all bins
};

// Warp 0 scans NB weights (bin 0 ranks first) and finds the crossing of `lim`.
// Every thread must call; the result is published in *out after the barrier.
template <typename W>
__device__ __forceinline__ void find_crossing(const W* w, u64 lim, Cross* out) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < 32) {
    constexpr int PER = NB / 32;
    u64 loc[PER];
    u64 s = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      loc[i] = (u64)w[lane * PER + i];
      s += loc[i];
    }
    const u64 incl = warp_incl_scan_u64(s, lane);
    const u64 excl = incl - s;
    const u64 total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      out->bin = -1;
      out->above = total;
      out->w = 0;
      out->total = total;
    }
    __syncwarp();
    if (excl <= lim && lim < incl) {
      u64 c = excl;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        if (c + loc[i] > lim) {
          out->bin = lane * PER + i;
          out->above = c;
          out->w = loc[i];
          break;
        }
        c += loc[i];
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// shared memory
// ---------------------------------------------------------------------------
struct alignas(16) StatX {  // per-CTA row statistics exchanged across the cluster
  float mx;
  int32_t amax;
  int32_t nan_id;
  uint32_t nfin;
  uint32_t pinf;
  uint32_t status;
  uint32_t pad[2];
};

template <int CS, int NCH>
struct alignas(16) Shared {
  // prologue results
  int32_t mono;
  int32_t mono_hi;
  uint32_t allow;
  int32_t grammar_on;
  float t_row;
  float t_rcp;
  float u;
  uint32_t status;
  int32_t n_uniq;
  int32_t nc;           // local candidate count
  int32_t token;
  int32_t red_i[2];
  float tk;
  uint32_t nsurv;
  float cut_x;
  int32_t cut_id;
  u64 qtot;
  u64 qkept;
  Cross cr;
  StatX stat;
  u64 cta_mass;         // kept mass of this CTA's tile (dense draw exchange)
  // per-warp partials
  float wf[32];
  int32_t wi[32];
  int32_t wi2[32];
  uint32_t wu[32];
  uint32_t wu2[32];
  u64 wl[32 * NCH];
  // histograms (local; merged copies when CS > 1)
  uint32_t hcnt[NB];
  u64 hmass[NB];
  uint32_t hcnt_m[CS > 1 ? NB : 1];
  u64 hmass_m[CS > 1 ? NB : 1];
  // candidate lists (local; merged when CS > 1)
  float cx[CAP];
  int32_t cid[CAP];
  uint32_t cq[CAP];
  float mcx[CS > 1 ? CAP : 1];
  int32_t mcid[CS > 1 ? CAP : 1];
  uint32_t mcq[CS > 1 ? CAP : 1];
  uint8_t ckeep[CAP];
};

// Host-derived constants of one launch.
struct Derived {
  int64_t second;    // rows between a first-half row and its partner
  int32_t pen_on;
  int32_t vec_ok;    // 16-byte loads of logits allowed
  int32_t cls_vec;   // vector loads of grammar_class_of allowed
  int32_t out_vec;   // float4 stores of out_scores allowed
  int32_t lp_vec;    // float4 stores of out_logprobs allowed
  int32_t topk_on;
  int32_t topp_on;
  int32_t ids_len;
  float temp_rcp;
  float cond_rcp[MTR_MAX_COND_TEMPS];
  float col_rcp[MTR_MAX_COL_TEMP_RANGES];
};

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <typename Tin, int THREADS, int EPT, int CS>
__global__ void __launch_bounds__(THREADS, (THREADS <= 256 ? 2 : 1))
    sampler_kernel(const __grid_constant__ MtrSamplerArgs a, const __grid_constant__ Derived dv) {
  using E = Elem<Tin>;
  constexpr int VEC = E::VEC;
  constexpr int NCH = EPT / VEC;
  constexpr int TILE = THREADS * EPT;
  constexpr int NW = THREADS / 32;
  static_assert(EPT % VEC == 0, "EPT must be a multiple of the vector width");
  static_assert(THREADS >= NB && THREADS >= CAP, "one thread per bin / candidate");

  __shared__ Shared<CS, NCH> sm;
  extern __shared__ __align__(16) uint8_t dsm[];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int crank = Clu<CS>::rank();
  const int64_t row = (int64_t)(blockIdx.x / CS);
  const int base = crank * TILE;
  const int V = a.vocab;
  const int L = a.input_ids ? dv.ids_len : 0;
  const float NEG = neg_inf();

  auto id_of = [&](int k) -> int { return base + ((k / VEC) * THREADS + tid) * VEC + (k % VEC); };

  // ------------------------------------------------------------ prologue
  int32_t mono = -1;
  if (a.mono_mode == MTR_MONO_SCAN) {
    int lts = -1, lsos = -1;
    for (int i = tid; i < L; i += THREADS) {
      const int64_t t = load_id(a, row, i);
      if (t >= a.ts_start && t < a.ts_end) lts = i;
      if (is_sos(a, t)) lsos = i;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lts = max(lts, __shfl_xor_sync(0xffffffffu, lts, o));
      lsos = max(lsos, __shfl_xor_sync(0xffffffffu, lsos, o));
    }
    if (lane == 0) {
      sm.wi[warp] = lts;
      sm.wi2[warp] = lsos;
    }
    __syncthreads();
    if (tid == 0) {
      int m1 = -1, m2 = -1;
      for (int w = 0; w < NW; ++w) {
        m1 = max(m1, sm.wi[w]);
        m2 = max(m2, sm.wi2[w]);
      }
      sm.red_i[0] = (m1 != -1 && m1 > m2) ? (int32_t)(load_id(a, row, m1) - a.ts_start) : -1;
    }
    __syncthreads();
    mono = sm.red_i[0];
  }
  if (tid == 0) {
    uint32_t status = 0;
    if (a.mono_mode == MTR_MONO_STATE) {
      mono = a.mono_state[row];
      if ((a.flags & MTR_FLAG_MONO_UPDATE_FROM_IDS) && L > 0) mono = mono_update(a, mono, load_id(a, row, L - 1));
    }
    sm.mono = mono;
    sm.mono_hi = mono >= 0 ? (int32_t)min((int64_t)a.ts_end, (int64_t)a.ts_start + mono) : -1;
    // grammar row of the previous token
    uint32_t allow = 0xffffffffu;
    int gon = 0;
    if (a.grammar_class_of) {
      int64_t prev = -1;
      if (a.flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) prev = L > 0 ? load_id(a, row, L - 1) : -1;
      else if (a.prev_token) prev = a.prev_token[row];
      if (prev >= V) status |= MTR_ROW_BAD_ID;
      if (prev >= 0 && prev < V) {
        const uint32_t c = __ldg(a.grammar_class_of + prev);
        if (c < (uint32_t)a.grammar_n_classes) {
          gon = 1;
          allow = __ldg(a.grammar_allow + c);
        } else {
          status |= MTR_ROW_BAD_ID;
        }
      }
    }
    sm.allow = allow;
    sm.grammar_on = gon;
    // per-row temperature
    float t = a.temperature, y = dv.temp_rcp;
    if (a.temp_mode == MTR_TEMP_ROW_CONDITIONAL) {
      for (int c = 0; c < a.n_cond; ++c) {
        const int off = a.cond_offset[c];
        if (off < 1 || L < off) continue;
        const int64_t tok = load_id(a, row, L - off);
        if (tok >= 0 && tok < V && ((__ldg(a.cond_token_bits[c] + (tok >> 5)) >> (tok & 31)) & 1u)) {
          t = a.cond_temperature[c];
          y = dv.cond_rcp[c];
          break;
        }
      }
    }
    sm.t_row = t;
    sm.t_rcp = y;
    float u = 0.0f;
    if (a.select_mode == MTR_SELECT_SAMPLE) {
      u = a.uniforms[row];
      if (!(u >= 0.0f)) {
        u = 0.0f;
        status |= MTR_ROW_BAD_UNIFORM;
      } else if (u >= 1.0f) {
        u = 0x1.fffffep-1f;
        status |= MTR_ROW_BAD_UNIFORM;
      }
    }
    sm.u = u;
    sm.status = status;
    sm.n_uniq = 0;
    sm.nc = 0;
    sm.token = -1;
  }

  // ------------------------------------------------------------ load
  const Tin* r1 = (const Tin*)a.logits + row * a.logits_row_stride;
  const Tin* r2 = r1 + dv.second * a.logits_row_stride;
  float x[EPT];
  if (dv.vec_ok) {
    uint4 ra[NCH], rb[NCH];
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int id0 = base + (j * THREADS + tid) * VEC;
      ra[j] = make_uint4(0u, 0u, 0u, 0u);
      rb[j] = make_uint4(0u, 0u, 0u, 0u);
      if (id0 < V) {
        ra[j] = __ldcs((const uint4*)(r1 + id0));
        if (a.cfg_enabled) rb[j] = __ldcs((const uint4*)(r2 + id0));
      }
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int k = j * VEC + e;
        const float va = E::get(ra[j], e);
        float v = va;
        if (a.cfg_enabled) {
          const float vb = E::get(rb[j], e);
          v = __fadd_rn(vb, __fmul_rn(__fsub_rn(va, vb), a.cfg_scale));
        }
        x[k] = (id_of(k) < V) ? v : NEG;
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const int id = id_of(k);
      float v = NEG;
      if (id < V) {
        const float va = E::one(r1, id);
        v = va;
        if (a.cfg_enabled) {
          const float vb = E::one(r2, id);
          v = __fadd_rn(vb, __fmul_rn(__fsub_rn(va, vb), a.cfg_scale));
        }
      }
      x[k] = v;
    }
  }
  __syncthreads();  // prologue scalars visible

  // ------------------------------------------------------------ mask chain
  {
    const int mono_hi = sm.mono_hi;
    const int ts0 = a.ts_start, ts1 = a.ts_end;
    const bool bias_on = a.timeshift_bias != 0.0f;
    const bool gon = sm.grammar_on != 0;
    const uint32_t allow = sm.allow;
    const uint32_t ncls = (uint32_t)a.grammar_n_classes;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int id0 = base + (j * THREADS + tid) * VEC;
      uint8_t cls[VEC];
      if (gon) {
        if (dv.cls_vec && id0 < V) {
          if constexpr (VEC == 8) {
            const uint2 w = __ldg((const uint2*)(a.grammar_class_of + id0));
#pragma unroll
            for (int e = 0; e < 8; ++e) cls[e] = (uint8_t)(((e < 4 ? w.x : w.y) >> (8 * (e & 3))) & 0xffu);
          } else {
            const uint32_t w = __ldg((const uint32_t*)(a.grammar_class_of + id0));
#pragma unroll
            for (int e = 0; e < VEC; ++e) cls[e] = (uint8_t)((w >> (8 * e)) & 0xffu);
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) cls[e] = (id0 + e < V) ? __ldg(a.grammar_class_of + id0 + e) : 0;
        }
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int k = j * VEC + e;
        const int id = id0 + e;
        float v = x[k];
        if (id >= ts0 && id < mono_hi) v = NEG;
        if (bias_on && id >= ts0 && id < ts1) v = __fadd_rn(v, a.timeshift_bias);
        if (gon) {
          const uint32_t c = cls[e];
          if (!(c < ncls && ((allow >> c) & 1u))) v = NEG;
        }
        if (id < V) x[k] = v;
      }
    }
  }

  // ------------------------------------------------------------ penalties
  if (dv.pen_on) {
    float* xs = (float*)dsm;
    uint32_t* cnt = (uint32_t*)(xs + TILE);
    uint16_t* uniq = (uint16_t*)(cnt + TILE);
    for (int i = tid; i < TILE; i += THREADS) cnt[i] = 0u;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int li0 = (j * THREADS + tid) * VEC;
#pragma unroll
      for (int e = 0; e < VEC; e += 4)
        *(float4*)(xs + li0 + e) = make_float4(x[j * VEC + e], x[j * VEC + e + 1], x[j * VEC + e + 2], x[j * VEC + e + 3]);
    }
    __syncthreads();
    uint32_t bad = 0;
    for (int i = a.penalty_start + tid; i < L; i += THREADS) {
      const int64_t t = load_id(a, row, i);
      if (t < 0 || t >= V) {
        bad = 1;
        continue;
      }
      if (t >= base && t < base + TILE) {
        const int li = (int)(t - base);
        if (atomicAdd(&cnt[li], 1u) == 0u) uniq[atomicAdd(&sm.n_uniq, 1)] = (uint16_t)li;
      }
    }
    if (bad) atomicOr(&sm.status, MTR_ROW_BAD_ID);
    __syncthreads();
    const int nu = sm.n_uniq;
    const float rp = a.repetition_penalty, fp = a.frequency_penalty, pp = a.presence_penalty;
    for (int i = tid; i < nu; i += THREADS) {
      const int li = uniq[i];
      const uint32_t c = cnt[li];
      float v = xs[li];
      if (rp != 1.0f) v = v < 0.0f ? __fmul_rn(v, rp) : __fdiv_rn(v, rp);
      if (fp != 0.0f) v = __fsub_rn(v, __fmul_rn(fp, (float)c));
      if (pp != 0.0f) v = __fsub_rn(v, pp);
      xs[li] = v;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int li0 = (j * THREADS + tid) * VEC;
#pragma unroll
      for (int e = 0; e < VEC; e += 4) {
        const float4 f = *(const float4*)(xs + li0 + e);
        x[j * VEC + e] = f.x;
        x[j * VEC + e + 1] = f.y;
        x[j * VEC + e + 2] = f.z;
        x[j * VEC + e + 3] = f.w;
      }
    }
  }

  // ------------------------------------------------------------ temperature
  if (a.temp_mode == MTR_TEMP_COLUMN_RANGES) {
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const int id = id_of(k);
      float t = a.temperature, y = dv.temp_rcp;
      for (int r = a.n_col_ranges - 1; r >= 0; --r) {
        if (id >= a.col_start[r] && id < a.col_end[r]) {
          t = a.col_temperature[r];
          y = dv.col_rcp[r];
        }
      }
      if (t != 1.0f) x[k] = div_by(x[k], t, y);
    }
  } else {
    const float t = sm.t_row, y = sm.t_rcp;
    if (t != 1.0f) {
#pragma unroll
      for (int k = 0; k < EPT; ++k) x[k] = div_by(x[k], t, y);
    }
  }

  // ------------------------------------------------------------ row statistics
  float gmax;
  int32_t gamax, gnan;
  uint32_t gnfin, gstatus;
  bool gpinf;
  {
    float lm = NEG;
    int32_t la = NO_ID, ln = NO_ID;
    uint32_t nf = 0, pinf = 0;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const float v = x[k];
      const int id = id_of(k);
      if (v != v) {
        ln = min(ln, id);
      } else {
        if (v > lm) {
          lm = v;
          la = id;
        }
        if (v == pos_inf()) pinf = 1;
        if (finite_val(v)) ++nf;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, lm, o);
      const int32_t oa = __shfl_xor_sync(0xffffffffu, la, o);
      if (om > lm || (om == lm && oa < la)) {
        lm = om;
        la = oa;
      }
      ln = min(ln, __shfl_xor_sync(0xffffffffu, ln, o));
      nf += __shfl_xor_sync(0xffffffffu, nf, o);
      pinf |= __shfl_xor_sync(0xffffffffu, pinf, o);
    }
    if (lane == 0) {
      sm.wf[warp] = lm;
      sm.wi[warp] = la;
      sm.wi2[warp] = ln;
      sm.wu[warp] = nf;
      sm.wu2[warp] = pinf;
    }
    __syncthreads();
    if (tid == 0) {
      float m = NEG;
      int32_t am = NO_ID, an = NO_ID;
      uint32_t n = 0, p = 0;
      for (int w = 0; w < NW; ++w) {
        if (sm.wf[w] > m || (sm.wf[w] == m && sm.wi[w] < am)) {
          m = sm.wf[w];
          am = sm.wi[w];
        }
        an = min(an, sm.wi2[w]);
        n += sm.wu[w];
        p |= sm.wu2[w];
      }
      sm.stat.mx = m;
      sm.stat.amax = am;
      sm.stat.nan_id = an;
      sm.stat.nfin = n;
      sm.stat.pinf = p;
      sm.stat.status = sm.status;
    }
    Clu<CS>::sync();
    gmax = NEG;
    gamax = NO_ID;
    gnan = NO_ID;
    gnfin = 0;
    gpinf = false;
    gstatus = 0;
#pragma unroll
    for (int r = 0; r < CS; ++r) {
      const StatX s = *Clu<CS>::at(&sm.stat, r);
      if (s.mx > gmax || (s.mx == gmax && s.amax < gamax)) {
        gmax = s.mx;
        gamax = s.amax;
      }
      gnan = min(gnan, s.nan_id);
      gnfin += s.nfin;
      gpinf |= s.pinf != 0;
      gstatus |= s.status;
    }
  }
  const bool nonfinite = gnan != NO_ID || gpinf;
  const bool all_masked = !nonfinite && gmax == NEG;
  if (nonfinite) gstatus |= MTR_ROW_NONFINITE;
  if (all_masked) gstatus |= MTR_ROW_ALL_MASKED;
  const bool clean = !nonfinite && !all_masked;
  const int sel = a.select_mode;
  const bool force_radix = (a.flags & MTR_FLAG_FORCE_RADIX) != 0;

  // selection state
  float tk = NEG;           // top-k threshold (keep x >= tk)
  bool topp_cut = false;    // keep also requires canonical <= (cut_x, cut_id)
  float cut_x = 0.0f;
  int32_t cut_id = NO_ID;
  u64 qkept = 0;
  int32_t token = -1;
  int owner = 0;            // cluster rank that writes the row's scalar outputs
  uint32_t q[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) q[k] = 0u;
  const bool want_lp = a.out_logprobs != nullptr;
  const bool need_mass = clean && (sel == MTR_SELECT_SAMPLE || want_lp || (sel == MTR_SELECT_NONE && dv.topp_on));

  // radix fallback: finds v with W(> v) <= lim < W(>= v) among candidates
  // (pred), descending by key, weights wt; above0 = weight ranked above all
  // candidates.  Returns v, W(> v) and the count / weight of key == v.
  auto radix_select = [&](auto pred, auto keyf, auto wt, u64 lim, u64 above0, uint32_t& out_key, u64& out_above,
                          uint32_t& out_cnt, u64& out_w) {
    uint32_t prefix = 0, mask = 0;
    u64 above = above0;
    u64 lastw = 0;
    uint32_t lastc = 0;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
      Clu<CS>::sync();  // previous readers of the histograms are done
      for (int i = tid; i < NB; i += THREADS) {
        sm.hcnt[i] = 0u;
        sm.hmass[i] = 0ull;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        if (pred(k)) {
          const uint32_t key = keyf(k);
          if ((key & mask) == prefix) {
            const int b = 255 - (int)((key >> shift) & 255u);
            atomicAdd(&sm.hcnt[b], 1u);
            atomicAdd(&sm.hmass[b], (u64)wt(k));
          }
        }
      }
      Clu<CS>::sync();
      const uint32_t* hc = sm.hcnt;
      const u64* hm = sm.hmass;
      if constexpr (CS > 1) {
        for (int i = tid; i < NB; i += THREADS) {
          uint32_t c = 0;
          u64 m = 0;
#pragma unroll
          for (int r = 0; r < CS; ++r) {
            c += Clu<CS>::at(sm.hcnt, r)[i];
            m += Clu<CS>::at(sm.hmass, r)[i];
          }
          sm.hcnt_m[i] = c;
          sm.hmass_m[i] = m;
        }
        __syncthreads();
        hc = sm.hcnt_m;
        hm = sm.hmass_m;
      }
      find_crossing(hm, lim - above, &sm.cr);
      const int b = max(sm.cr.bin, 0);  // a crossing exists: above <= lim < above + candidates
      const uint32_t d = 255u - (uint32_t)b;
      prefix |= d << shift;
      mask |= 255u << shift;
      above += sm.cr.above;
      lastw = sm.cr.w;
      lastc = hc[b];
      __syncthreads();
    }
    out_key = prefix;
    out_above = above;
    out_cnt = lastc;
    out_w = lastw;
  };

  // merge the per-CTA candidate lists into (mcx, mcid, mcq); returns the total
  auto merge_lists = [&](int& n_total, const float*& lx, const int32_t*& lid, const uint32_t*& lq) {
    Clu<CS>::sync();
    if constexpr (CS == 1) {
      n_total = sm.nc;
      lx = sm.cx;
      lid = sm.cid;
      lq = sm.cq;
    } else {
      int tot = 0;
      int offs[CS];
#pragma unroll
      for (int r = 0; r < CS; ++r) {
        offs[r] = tot;
        tot += *Clu<CS>::at(&sm.nc, r);
      }
      n_total = tot;
      if (tot <= CAP) {
#pragma unroll
        for (int r = 0; r < CS; ++r) {
          const int n = *Clu<CS>::at(&sm.nc, r);
          const float* rx = Clu<CS>::at(sm.cx, r);
          const int32_t* ri = Clu<CS>::at(sm.cid, r);
          const uint32_t* rq = Clu<CS>::at(sm.cq, r);
          for (int i = tid; i < n; i += THREADS) {
            sm.mcx[offs[r] + i] = rx[i];
            sm.mcid[offs[r] + i] = ri[i];
            sm.mcq[offs[r] + i] = rq[i];
          }
        }
      }
      __syncthreads();
      lx = sm.mcx;
      lid = sm.mcid;
      lq = sm.mcq;
    }
  };

  // ------------------------------------------------------------ selection
  if (clean && sel == MTR_SELECT_ARGMAX) {
    token = gamax;
  } else if (clean && sel != MTR_SELECT_ARGMAX) {
    // ---------------- top-k
    uint32_t nsurv = gnfin;
    const bool topk_on = dv.topk_on && (uint32_t)a.top_k < gnfin;
    if (topk_on) {
      const u64 lim = (u64)(a.top_k - 1);
      for (int i = tid; i < NB; i += THREADS) sm.hcnt[i] = 0u;
      if (tid == 0) sm.nc = 0;
      __syncthreads();
#pragma unroll
      for (int k = 0; k < EPT; ++k)
        if (finite_val(x[k])) atomicAdd(&sm.hcnt[dbin(gmax, x[k])], 1u);
      Clu<CS>::sync();
      const uint32_t* hc = sm.hcnt;
      if constexpr (CS > 1) {
        for (int i = tid; i < NB; i += THREADS) {
          uint32_t c = 0;
#pragma unroll
          for (int r = 0; r < CS; ++r) c += Clu<CS>::at(sm.hcnt, r)[i];
          sm.hcnt_m[i] = c;
        }
        __syncthreads();
        hc = sm.hcnt_m;
      }
      find_crossing(hc, lim, &sm.cr);
      const int bstar = max(sm.cr.bin, 0);  // k - 1 < finite count, so a crossing exists
      const u64 c_above = sm.cr.above;
      const u64 n_c = sm.cr.w;
      if (n_c <= (u64)CAP && !force_radix) {
#pragma unroll
        for (int k = 0; k < EPT; ++k)
          if (finite_val(x[k]) && dbin(gmax, x[k]) == bstar) sm.cx[atomicAdd(&sm.nc, 1)] = x[k];
        int n;
        const float* lx;
        const int32_t* lid;
        const uint32_t* lq;
        merge_lists(n, lx, lid, lq);
        if (tid < n) {
          const float xi = lx[tid];
          uint32_t gt = 0, ge = 0;
          for (int jj = 0; jj < n; ++jj) {
            const float xj = lx[jj];
            gt += xj > xi;
            ge += xj >= xi;
          }
          if (c_above + gt <= lim && lim < c_above + ge) {
            sm.tk = xi;
            sm.nsurv = (uint32_t)(c_above + ge);
          }
        }
        __syncthreads();
        tk = sm.tk;
        nsurv = sm.nsurv;
      } else {
        uint32_t key, cntv;
        u64 abv, wv;
        radix_select([&](int k) { return finite_val(x[k]) && dbin(gmax, x[k]) == bstar; },
                     [&](int k) { return fkey(x[k]); }, [&](int) { return 1u; }, lim, c_above, key, abv, cntv, wv);
        tk = key2f(key);
        nsurv = (uint32_t)(abv + wv);
        gstatus |= MTR_ROW_SLOW_PATH;
      }
#pragma unroll
      for (int k = 0; k < EPT; ++k)
        if (x[k] < tk) x[k] = NEG;
    }

    // ---------------- top-p and the draw
    if (need_mass) {
      const bool topp_on = dv.topp_on != 0;
      const float u = sm.u;
      if (nsurv <= (uint32_t)CAP && !force_radix) {
        // compact path: every survivor in one list
        Clu<CS>::sync();
        if (tid == 0) sm.nc = 0;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < EPT; ++k) {
          if (finite_val(x[k])) {
            const int s = atomicAdd(&sm.nc, 1);
            sm.cx[s] = x[k];
            sm.cid[s] = id_of(k);
            sm.cq[s] = expfx(__fsub_rn(x[k], gmax));
          }
        }
        int n;
        const float* lx;
        const int32_t* lid;
        const uint32_t* lq;
        merge_lists(n, lx, lid, lq);
        float xi = 0.0f;
        int32_t ii = 0;
        u64 qi = 0, ai = 0, tot = 0;
        if (tid < n) {
          xi = lx[tid];
          ii = lid[tid];
          qi = lq[tid];
          for (int jj = 0; jj < n; ++jj) {
            const float xj = lx[jj];
            const u64 qj = lq[jj];
            tot += qj;
            if (xj > xi || (xj == xi && lid[jj] < ii)) ai += qj;
          }
          if (tid == 0) sm.qtot = tot;
        }
        __syncthreads();
        tot = sm.qtot;
        bool kept = tid < n;
        if (topp_on) {
          const double P = __dmul_rn((double)a.top_p, (double)tot);
          const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
          kept = kept && ai <= plim;
          if (kept && ai + qi > plim) {
            sm.cut_x = xi;
            sm.cut_id = ii;
            sm.qkept = ai + qi;
          }
        } else if (tid == 0) {
          sm.qkept = tot;
        }
        if (tid < CAP) sm.ckeep[tid] = kept ? 1 : 0;
        __syncthreads();
        qkept = sm.qkept;
        if (topp_on) {
          topp_cut = true;
          cut_x = sm.cut_x;
          cut_id = sm.cut_id;
          if (tid < n && xi == cut_x && ii > cut_id) atomicOr(&sm.status, MTR_ROW_TIE_AT_CUT);
        }
        if (sel == MTR_SELECT_SAMPLE) {
          const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
          if (kept) {
            u64 ci = 0;
            for (int jj = 0; jj < n; ++jj)
              if (sm.ckeep[jj] && lid[jj] <= ii) ci += lq[jj];
            if (ci > R && ci - qi <= R) sm.token = ii;
          }
        }
        __syncthreads();
        gstatus |= sm.status & MTR_ROW_TIE_AT_CUT;
        token = sm.token;
      } else {
        // dense path: per-element fixed-point probabilities
#pragma unroll
        for (int k = 0; k < EPT; ++k) q[k] = finite_val(x[k]) ? expfx(__fsub_rn(x[k], gmax)) : 0u;
        if (topp_on) {
          Clu<CS>::sync();
          for (int i = tid; i < NB; i += THREADS) sm.hmass[i] = 0ull;
          if (tid == 0) sm.nc = 0;
          __syncthreads();
#pragma unroll
          for (int k = 0; k < EPT; ++k)
            if (q[k]) atomicAdd(&sm.hmass[dbin(gmax, x[k])], (u64)q[k]);
          Clu<CS>::sync();
          const u64* hm = sm.hmass;
          if constexpr (CS > 1) {
            for (int i = tid; i < NB; i += THREADS) {
              u64 m = 0;
#pragma unroll
              for (int r = 0; r < CS; ++r) m += Clu<CS>::at(sm.hmass, r)[i];
              sm.hmass_m[i] = m;
            }
            __syncthreads();
            hm = sm.hmass_m;
          }
          // total first, then the crossing of plim
          find_crossing(hm, ~0ull - 1ull, &sm.cr);
          const u64 tot = sm.cr.total;
          const double P = __dmul_rn((double)a.top_p, (double)tot);
          const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
          __syncthreads();
          find_crossing(hm, plim, &sm.cr);
          const int bstar = max(sm.cr.bin, 0);  // plim < total since top_p < 1
          const u64 w_above = sm.cr.above;
#pragma unroll
          for (int k = 0; k < EPT; ++k) {
            if (q[k] && dbin(gmax, x[k]) == bstar) {
              const int s = atomicAdd(&sm.nc, 1);
              if (s < CAP) {
                sm.cx[s] = x[k];
                sm.cid[s] = id_of(k);
                sm.cq[s] = q[k];
              }
            }
          }
          int n;
          const float* lx;
          const int32_t* lid;
          const uint32_t* lq;
          // per-CTA overflow is detected through the merged total
          merge_lists(n, lx, lid, lq);
          if (n <= CAP && !force_radix) {
            if (tid < n) {
              const float xi = lx[tid];
              const int32_t ii = lid[tid];
              const u64 qi = lq[tid];
              u64 ai = w_above;
              for (int jj = 0; jj < n; ++jj) {
                const float xj = lx[jj];
                if (xj > xi || (xj == xi && lid[jj] < ii)) ai += lq[jj];
              }
              if (ai <= plim && ai + qi > plim) {
                sm.cut_x = xi;
                sm.cut_id = ii;
                sm.qkept = ai + qi;
              }
            }
            __syncthreads();
            cut_x = sm.cut_x;
            cut_id = sm.cut_id;
            qkept = sm.qkept;
            if (tid < n && lx[tid] == cut_x && lid[tid] > cut_id) atomicOr(&sm.status, MTR_ROW_TIE_AT_CUT);
            __syncthreads();
            gstatus |= sm.status & MTR_ROW_TIE_AT_CUT;
          } else {
            uint32_t key, cntv;
            u64 abv, wv;
            radix_select([&](int k) { return q[k] != 0u && dbin(gmax, x[k]) == bstar; },
                         [&](int k) { return fkey(x[k]); }, [&](int k) { return q[k]; }, plim, w_above, key, abv,
                         cntv, wv);
            const float vstar = key2f(key);
            const u64 qv = wv / (u64)cntv;  // members of the tie group share q
            u64 nkeep = (plim - abv) / qv + 1ull;
            if (nkeep > cntv) nkeep = cntv;
            cut_x = vstar;
            cut_id = NO_ID;
            if (nkeep < cntv) {
              uint32_t ikey, c2;
              u64 a2, w2;
              radix_select([&](int k) { return q[k] != 0u && x[k] == vstar; },
                           [&](int k) { return ~(uint32_t)id_of(k); }, [&](int) { return 1u; }, nkeep - 1ull, 0ull,
                           ikey, a2, c2, w2);
              cut_id = (int32_t)(~ikey);
              gstatus |= MTR_ROW_TIE_AT_CUT;
            }
            qkept = abv + nkeep * qv;
            gstatus |= MTR_ROW_SLOW_PATH;
          }
          topp_cut = true;
        } else {
          // kept mass = all survivors
          u64 s = 0;
#pragma unroll
          for (int k = 0; k < EPT; ++k) s += q[k];
          s = warp_sum_u64(s);
          if (lane == 0) sm.wl[warp] = s;
          __syncthreads();
          if (tid == 0) {
            u64 t = 0;
            for (int w = 0; w < NW; ++w) t += sm.wl[w];
            sm.cta_mass = t;
          }
          Clu<CS>::sync();
          u64 t = 0;
#pragma unroll
          for (int r = 0; r < CS; ++r) t += *Clu<CS>::at(&sm.cta_mass, r);
          qkept = t;
        }
        // drop the removed tail from q (kept = survivors up to the cut)
        if (topp_cut) {
#pragma unroll
          for (int k = 0; k < EPT; ++k) {
            const float v = x[k];
            const bool kp = v > cut_x || (v == cut_x && id_of(k) <= cut_id);
            if (!kp) q[k] = 0u;
          }
        }
        if (sel == MTR_SELECT_SAMPLE) {
          const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
          // per-chunk kept mass of this thread, then chunk totals of the CTA
          u64 cs[NCH];
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            u64 s = 0;
#pragma unroll
            for (int e = 0; e < VEC; ++e) s += q[j * VEC + e];
            cs[j] = s;
          }
          Clu<CS>::sync();  // wl / cta_mass free for reuse
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            const u64 s = warp_sum_u64(cs[j]);
            if (lane == 0) sm.wl[j * 32 + warp] = s;
          }
          __syncthreads();
          u64 ctot[NCH];
          u64 cta = 0;
#pragma unroll
          for (int j = 0; j < NCH; ++j) {
            u64 s = 0;
            for (int w = 0; w < NW; ++w) s += sm.wl[j * 32 + w];
            ctot[j] = s;
            cta += s;
          }
          if (tid == 0) sm.cta_mass = cta;
          Clu<CS>::sync();
          // which CTA holds the draw (R < qkept = sum of the CTA masses)
          u64 before = 0;
          int cstar = -1;
#pragma unroll
          for (int r = 0; r < CS; ++r) {
            const u64 m = *Clu<CS>::at(&sm.cta_mass, r);
            if (cstar < 0) {
              if (R < before + m) cstar = r;
              else before += m;
            }
          }
          if (cstar < 0) cstar = CS - 1;
          owner = cstar;
          if (crank == cstar) {
            u64 rr = R - before;
            int jstar = -1;
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
              if (jstar < 0) {
                if (rr < ctot[j]) jstar = j;
                else rr -= ctot[j];
              }
            }
            if (jstar < 0) jstar = NCH - 1;
            u64 mine = 0;
#pragma unroll
            for (int j = 0; j < NCH; ++j)
              if (j == jstar) mine = cs[j];
            // exclusive scan of `mine` over the CTA
            const u64 incl = warp_incl_scan_u64(mine, lane);
            if (lane == 31) sm.wl[warp] = incl;
            __syncthreads();
            u64 wbefore = 0;
            for (int w = 0; w < warp; ++w) wbefore += sm.wl[w];
            const u64 excl = wbefore + incl - mine;
            if (mine != 0 && excl <= rr && rr < excl + mine) {
              u64 c = excl;
              bool done = false;
#pragma unroll
              for (int j = 0; j < NCH; ++j) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  const int k = j * VEC + e;
                  if (j == jstar && !done) {
                    c += q[k];
                    if (c > rr) {
                      sm.token = id_of(k);
                      done = true;
                    }
                  }
                }
              }
            }
            __syncthreads();
            token = sm.token;
          }
        }
      }
    }
  }
  if (!clean && sel == MTR_SELECT_ARGMAX) token = gnan != NO_ID ? gnan : (gmax == NEG ? 0 : gamax);
  if (!clean && sel == MTR_SELECT_SAMPLE) token = (int32_t)a.pad_id;

  // ------------------------------------------------------------ epilogue
  // processed scores: survivors of top-k and top-p; unfiltered for argmax
  const bool filter_out = clean && sel != MTR_SELECT_ARGMAX;
  if (a.out_scores) {
    float* orow = a.out_scores + row * a.out_scores_row_stride;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int id0 = base + (j * THREADS + tid) * VEC;
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int k = j * VEC + e;
        float v = x[k];
        if (filter_out && topp_cut && !(v > cut_x || (v == cut_x && id0 + e <= cut_id))) v = NEG;
        o[e] = v;
      }
      if (dv.out_vec && id0 < V) {
#pragma unroll
        for (int e = 0; e < VEC; e += 4) __stcs((float4*)(orow + id0 + e), make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]));
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (id0 + e < V) orow[id0 + e] = o[e];
      }
    }
  }
  if (want_lp) {
    float* orow = a.out_logprobs + row * a.out_logprobs_row_stride;
    double lse = 0.0;
    if (clean) {
      if (sel == MTR_SELECT_ARGMAX || !need_mass) {
        // normaliser over every finite score
        u64 s = 0;
#pragma unroll
        for (int k = 0; k < EPT; ++k) s += finite_val(x[k]) ? expfx(__fsub_rn(x[k], gmax)) : 0u;
        s = warp_sum_u64(s);
        Clu<CS>::sync();
        if (lane == 0) sm.wl[warp] = s;
        __syncthreads();
        if (tid == 0) {
          u64 t = 0;
          for (int w = 0; w < NW; ++w) t += sm.wl[w];
          sm.cta_mass = t;
        }
        Clu<CS>::sync();
        u64 t = 0;
#pragma unroll
        for (int r = 0; r < CS; ++r) t += *Clu<CS>::at(&sm.cta_mass, r);
        qkept = t;
      }
      lse = log((double)qkept) - 31.0 * 0.69314718055994530942;
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int id0 = base + (j * THREADS + tid) * VEC;
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const int k = j * VEC + e;
        const float v = x[k];
        bool kp = finite_val(v);
        if (filter_out && topp_cut) kp = kp && (v > cut_x || (v == cut_x && id0 + e <= cut_id));
        o[e] = !clean ? __int_as_float(0x7fc00000) : kp ? (float)(((double)v - (double)gmax) - lse) : NEG;
      }
      if (dv.lp_vec && id0 < V) {
#pragma unroll
        for (int e = 0; e < VEC; e += 4) __stcs((float4*)(orow + id0 + e), make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]));
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (id0 + e < V) orow[id0 + e] = o[e];
      }
    }
  }

  // row scalars: one writer per row
  if (crank == owner && tid == 0) {
    int32_t m = sm.mono;
    if (sel != MTR_SELECT_NONE) {
      int64_t fin = token;
      if (a.unfinished) {
        const uint8_t uf = a.unfinished[row];
        if (!uf) fin = a.pad_id;
        a.unfinished[row] = (uint8_t)(uf && !is_eos(a, fin));
      }
      if (a.flags & MTR_FLAG_MONO_UPDATE_FROM_SAMPLE) m = mono_update(a, m, fin);
      if ((a.flags & MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE) && a.prev_token) a.prev_token[row] = (int32_t)fin;
      if (a.out_ids) a.out_ids[row] = fin;
    }
    if (a.mono_mode != MTR_MONO_OFF && a.mono_state) a.mono_state[row] = m;
    if (a.out_status) a.out_status[row] = gstatus;
  }
  if constexpr (CS > 1) cg::this_cluster().sync();  // no CTA leaves while its shared memory may be read
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Geo {
  int threads, ept, cs;
};

static Geo pick_geo(int V) {
  if (V <= 4096) return {256, 16, 1};
  if (V <= 8192) return {256, 16, 2};
  if (V <= 16384) return {256, 16, 4};
  if (V <= 32768) return {512, 16, 4};
  if (V <= 65536) return {512, 16, 8};
  return {1024, 16, 8};
}

static int dyn_smem_bytes(const Geo& g, bool pen) {
  if (!pen) return 0;
  const int tile = g.threads * g.ept;
  return tile * 4 + tile * 4 + tile * 2;
}

static thread_local int g_last_cuda_error = 0;

static bool bad_float(float v) { return !(v == v) || v == INFINITY || v == -INFINITY; }

static int validate(const MtrSamplerArgs* a) {
  if (!a) return MTR_ERR_NULL_ARG;
  if (a->abi_version != MTR_ABI_VERSION || a->struct_size != sizeof(MtrSamplerArgs)) return MTR_ERR_ABI;
  const uint32_t known = MTR_FLAG_MONO_UPDATE_FROM_IDS | MTR_FLAG_MONO_UPDATE_FROM_SAMPLE |
                         MTR_FLAG_GRAMMAR_PREV_FROM_IDS | MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE | MTR_FLAG_FORCE_RADIX;
  if (a->flags & ~known) return MTR_ERR_BAD_PARAM;
  if (a->num_rows < 0) return MTR_ERR_BAD_SHAPE;
  if (a->vocab < 1 || a->vocab > MTR_MAX_VOCAB) return MTR_ERR_BAD_SHAPE;
  if (a->num_rows == 0) return MTR_OK;
  if (!a->logits) return MTR_ERR_NULL_ARG;
  if (a->logits_dtype != MTR_DTYPE_F32 && a->logits_dtype != MTR_DTYPE_BF16 && a->logits_dtype != MTR_DTYPE_F16)
    return MTR_ERR_BAD_PARAM;
  const size_t esz = a->logits_dtype == MTR_DTYPE_F32 ? 4 : 2;
  if ((uintptr_t)a->logits % esz) return MTR_ERR_ALIGNMENT;
  if (a->logits_row_stride < a->vocab) return MTR_ERR_BAD_SHAPE;
  if (a->cfg_enabled) {
    if (bad_float(a->cfg_scale)) return MTR_ERR_BAD_PARAM;
  }
  if (a->cfg_second_offset < 0) return MTR_ERR_BAD_SHAPE;
  // history
  const bool ids_needed = a->mono_mode == MTR_MONO_SCAN || (a->flags & MTR_FLAG_MONO_UPDATE_FROM_IDS) ||
                          (a->flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) || a->temp_mode == MTR_TEMP_ROW_CONDITIONAL ||
                          a->repetition_penalty != 1.0f || a->frequency_penalty != 0.0f ||
                          a->presence_penalty != 0.0f;
  if (a->ids_len < 0 || a->ids_len > MTR_MAX_IDS_LEN) return MTR_ERR_BAD_SHAPE;
  if (a->input_ids) {
    if (a->ids_dtype != MTR_IDS_I64 && a->ids_dtype != MTR_IDS_I32) return MTR_ERR_BAD_PARAM;
    if ((uintptr_t)a->input_ids % (a->ids_dtype == MTR_IDS_I64 ? 8 : 4)) return MTR_ERR_ALIGNMENT;
    if (a->ids_row_stride < a->ids_len) return MTR_ERR_BAD_SHAPE;
  } else if (ids_needed && a->ids_len > 0) {
    return MTR_ERR_NULL_ARG;
  }
  if (a->penalty_start < 0 || (a->ids_len > 0 && a->penalty_start > a->ids_len)) return MTR_ERR_BAD_SHAPE;
  // monotonic
  if (a->mono_mode < MTR_MONO_OFF || a->mono_mode > MTR_MONO_SCAN) return MTR_ERR_BAD_PARAM;
  if (a->ts_start < 0 || a->ts_end < a->ts_start || a->ts_end > a->vocab) return MTR_ERR_BAD_SHAPE;
  if (a->n_sos < 0 || a->n_sos > MTR_MAX_SOS_IDS) return MTR_ERR_BAD_PARAM;
  if (a->mono_mode == MTR_MONO_STATE && !a->mono_state) return MTR_ERR_NULL_ARG;
  if ((uintptr_t)a->mono_state % 4) return MTR_ERR_ALIGNMENT;
  if (bad_float(a->timeshift_bias)) return MTR_ERR_BAD_PARAM;
  // grammar
  if (a->grammar_class_of) {
    if (!a->grammar_allow) return MTR_ERR_NULL_ARG;
    if (a->grammar_n_classes < 1 || a->grammar_n_classes > MTR_MAX_GRAMMAR_CLASSES) return MTR_ERR_BAD_PARAM;
    if (!(a->flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) && !a->prev_token) return MTR_ERR_NULL_ARG;
    if ((uintptr_t)a->grammar_allow % 4) return MTR_ERR_ALIGNMENT;
  }
  if ((uintptr_t)a->prev_token % 4) return MTR_ERR_ALIGNMENT;
  // penalties
  if (bad_float(a->repetition_penalty) || !(a->repetition_penalty > 0.0f)) return MTR_ERR_BAD_PARAM;
  if (bad_float(a->frequency_penalty) || bad_float(a->presence_penalty)) return MTR_ERR_BAD_PARAM;
  // temperature
  if (a->temp_mode < MTR_TEMP_SCALAR || a->temp_mode > MTR_TEMP_COLUMN_RANGES) return MTR_ERR_BAD_PARAM;
  if (bad_float(a->temperature) || !(a->temperature >= 0x1p-30f) || a->temperature > 0x1p30f) return MTR_ERR_BAD_PARAM;
  if (a->temp_mode == MTR_TEMP_ROW_CONDITIONAL) {
    if (a->n_cond < 0 || a->n_cond > MTR_MAX_COND_TEMPS) return MTR_ERR_BAD_PARAM;
    for (int c = 0; c < a->n_cond; ++c) {
      const float t = a->cond_temperature[c];
      if (bad_float(t) || !(t >= 0x1p-30f) || t > 0x1p30f) return MTR_ERR_BAD_PARAM;
      if (a->cond_offset[c] < 1) return MTR_ERR_BAD_PARAM;
      if (!a->cond_token_bits[c]) return MTR_ERR_NULL_ARG;
      if ((uintptr_t)a->cond_token_bits[c] % 4) return MTR_ERR_ALIGNMENT;
    }
  }
  if (a->temp_mode == MTR_TEMP_COLUMN_RANGES) {
    if (a->n_col_ranges < 0 || a->n_col_ranges > MTR_MAX_COL_TEMP_RANGES) return MTR_ERR_BAD_PARAM;
    for (int r = 0; r < a->n_col_ranges; ++r) {
      const float t = a->col_temperature[r];
      if (bad_float(t) || !(t >= 0x1p-30f) || t > 0x1p30f) return MTR_ERR_BAD_PARAM;
      if (a->col_start[r] < 0 || a->col_end[r] < a->col_start[r] || a->col_end[r] > a->vocab) return MTR_ERR_BAD_SHAPE;
    }
  }
  // selection
  if (a->select_mode < MTR_SELECT_NONE || a->select_mode > MTR_SELECT_SAMPLE) return MTR_ERR_BAD_PARAM;
  if (a->top_k < 0) return MTR_ERR_BAD_PARAM;
  if (!(a->top_p > 0.0f && a->top_p <= 1.0f)) return MTR_ERR_BAD_PARAM;
  if (a->top_p_mode != MTR_TOPP_HF && a->top_p_mode != MTR_TOPP_SAMPLE_FN) return MTR_ERR_BAD_PARAM;
  if (a->select_mode == MTR_SELECT_SAMPLE && !a->uniforms) return MTR_ERR_NULL_ARG;
  if (a->select_mode != MTR_SELECT_NONE && !a->out_ids) return MTR_ERR_NULL_ARG;
  if ((uintptr_t)a->uniforms % 4 || (uintptr_t)a->out_ids % 8) return MTR_ERR_ALIGNMENT;
  // outputs
  if (a->out_scores && a->out_scores_row_stride < a->vocab) return MTR_ERR_BAD_SHAPE;
  if (a->out_logprobs && a->out_logprobs_row_stride < a->vocab) return MTR_ERR_BAD_SHAPE;
  if ((uintptr_t)a->out_scores % 4 || (uintptr_t)a->out_logprobs % 4 || (uintptr_t)a->out_status % 4)
    return MTR_ERR_ALIGNMENT;
  if (a->n_eos < 0 || a->n_eos > MTR_MAX_EOS_IDS) return MTR_ERR_BAD_PARAM;
  if (a->n_eos_ranges < 0 || a->n_eos_ranges > MTR_MAX_EOS_RANGES) return MTR_ERR_BAD_PARAM;
  if (a->num_rows > (1 << 24)) return MTR_ERR_BAD_SHAPE;
  return MTR_OK;
}

static Derived derive(const MtrSamplerArgs& a) {
  Derived d;
  memset(&d, 0, sizeof(d));
  d.second = a.cfg_second_offset > 0 ? a.cfg_second_offset : a.num_rows;
  d.pen_on = (a.repetition_penalty != 1.0f || a.frequency_penalty != 0.0f || a.presence_penalty != 0.0f) &&
             a.input_ids != nullptr && a.ids_len > a.penalty_start;
  const int esz = a.logits_dtype == MTR_DTYPE_F32 ? 4 : 2;
  const int vec = 16 / esz;
  const uintptr_t lp = (uintptr_t)a.logits;
  d.vec_ok = (lp % 16 == 0) && ((a.logits_row_stride * esz) % 16 == 0) && (a.vocab % vec == 0);
  d.cls_vec = a.grammar_class_of && ((uintptr_t)a.grammar_class_of % vec == 0) && (a.vocab % vec == 0);
  d.out_vec = a.out_scores && ((uintptr_t)a.out_scores % 16 == 0) && ((a.out_scores_row_stride * 4) % 16 == 0) &&
              (a.vocab % vec == 0);
  d.lp_vec = a.out_logprobs && ((uintptr_t)a.out_logprobs % 16 == 0) &&
             ((a.out_logprobs_row_stride * 4) % 16 == 0) && (a.vocab % vec == 0);
  d.topk_on = a.select_mode != MTR_SELECT_ARGMAX && a.top_k > 0 && a.top_k < a.vocab;
  d.topp_on = a.select_mode != MTR_SELECT_ARGMAX && a.top_p < 1.0f;
  d.ids_len = a.input_ids ? a.ids_len : 0;
  d.temp_rcp = 1.0f / a.temperature;
  for (int c = 0; c < MTR_MAX_COND_TEMPS; ++c)
    d.cond_rcp[c] = (c < a.n_cond && a.cond_temperature[c] > 0.0f) ? 1.0f / a.cond_temperature[c] : 1.0f;
  for (int r = 0; r < MTR_MAX_COL_TEMP_RANGES; ++r)
    d.col_rcp[r] = (r < a.n_col_ranges && a.col_temperature[r] > 0.0f) ? 1.0f / a.col_temperature[r] : 1.0f;
  return d;
}

template <typename Tin, int TH, int EPT, int CS>
static cudaError_t launch_t(const MtrSamplerArgs& a, const Derived& d, int dyn, cudaStream_t s) {
  auto kern = sampler_kernel<Tin, TH, EPT, CS>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [&]() {
    const int max_dyn = 227 * 1024 - (int)sizeof(Shared<CS, EPT / Elem<Tin>::VEC>);
    attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn);
  });
  if (attr_err[dev] != cudaSuccess) return attr_err[dev];
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(a.num_rows * CS), 1, 1);
  cfg.blockDim = dim3(TH, 1, 1);
  cfg.dynamicSmemBytes = (size_t)dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (CS > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, a, d);
}

template <typename Tin>
static cudaError_t launch_dtype(const MtrSamplerArgs& a, const Derived& d, const Geo& g, int dyn, cudaStream_t s) {
  if (g.threads == 256 && g.cs == 1) return launch_t<Tin, 256, 16, 1>(a, d, dyn, s);
  if (g.threads == 256 && g.cs == 2) return launch_t<Tin, 256, 16, 2>(a, d, dyn, s);
  if (g.threads == 256 && g.cs == 4) return launch_t<Tin, 256, 16, 4>(a, d, dyn, s);
  if (g.threads == 512 && g.cs == 4) return launch_t<Tin, 512, 16, 4>(a, d, dyn, s);
  if (g.threads == 512 && g.cs == 8) return launch_t<Tin, 512, 16, 8>(a, d, dyn, s);
  return launch_t<Tin, 1024, 16, 8>(a, d, dyn, s);
}

}  // namespace mtr

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

int mtr_abi_version(void) { return MTR_ABI_VERSION; }

size_t mtr_args_size(void) { return sizeof(MtrSamplerArgs); }

int mtr_args_init(MtrSamplerArgs* a) {
  if (!a) return MTR_ERR_NULL_ARG;
  memset(a, 0, sizeof(*a));
  a->abi_version = MTR_ABI_VERSION;
  a->struct_size = (uint32_t)sizeof(MtrSamplerArgs);
  a->cfg_scale = 1.0f;
  a->repetition_penalty = 1.0f;
  a->temperature = 1.0f;
  a->top_p = 1.0f;
  a->mono_mode = MTR_MONO_OFF;
  a->select_mode = MTR_SELECT_NONE;
  a->pad_id = 0;
  return MTR_OK;
}

int mtr_sampler_validate(const MtrSamplerArgs* a) { return mtr::validate(a); }

int mtr_sampler_query(int32_t vocab, int32_t num_rows, int32_t with_penalties, MtrLaunchInfo* out) {
  if (!out) return MTR_ERR_NULL_ARG;
  if (vocab < 1 || vocab > MTR_MAX_VOCAB || num_rows < 0) return MTR_ERR_BAD_SHAPE;
  const mtr::Geo g = mtr::pick_geo(vocab);
  out->threads = g.threads;
  out->elems_per_thread = g.ept;
  out->cluster_size = g.cs;
  out->grid = num_rows * g.cs;
  out->dyn_smem_bytes = mtr::dyn_smem_bytes(g, with_penalties != 0);
  out->max_vocab = MTR_MAX_VOCAB;
  out->max_ids_len = MTR_MAX_IDS_LEN;
  out->candidate_cap = mtr::CAP;
  return MTR_OK;
}

int mtr_sampler_launch(const MtrSamplerArgs* a, void* stream) {
  const int v = mtr::validate(a);
  if (v != MTR_OK) return v;
  if (a->num_rows == 0) return MTR_OK;
  const mtr::Derived d = mtr::derive(*a);
  const mtr::Geo g = mtr::pick_geo(a->vocab);
  const int dyn = mtr::dyn_smem_bytes(g, d.pen_on != 0);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  switch (a->logits_dtype) {
    case MTR_DTYPE_F32: e = mtr::launch_dtype<float>(*a, d, g, dyn, s); break;
    case MTR_DTYPE_BF16: e = mtr::launch_dtype<__nv_bfloat16>(*a, d, g, dyn, s); break;
    default: e = mtr::launch_dtype<__half>(*a, d, g, dyn, s); break;
  }
  mtr::g_last_cuda_error = (int)e;
  return e == cudaSuccess ? MTR_OK : MTR_ERR_CUDA;
}

const char* mtr_status_string(int code) {
  switch (code) {
    case MTR_OK: return "MTR_OK";
    case MTR_ERR_NULL_ARG: return "MTR_ERR_NULL_ARG";
    case MTR_ERR_BAD_SHAPE: return "MTR_ERR_BAD_SHAPE";
    case MTR_ERR_BAD_PARAM: return "MTR_ERR_BAD_PARAM";
    case MTR_ERR_UNSUPPORTED: return "MTR_ERR_UNSUPPORTED";
    case MTR_ERR_ALIGNMENT: return "MTR_ERR_ALIGNMENT";
    case MTR_ERR_CUDA: return "MTR_ERR_CUDA";
    case MTR_ERR_ABI: return "MTR_ERR_ABI";
    default: return "MTR_ERR_UNKNOWN";
  }
}

int mtr_last_cuda_error(void) { return mtr::g_last_cuda_error; }

}  // extern "C"
