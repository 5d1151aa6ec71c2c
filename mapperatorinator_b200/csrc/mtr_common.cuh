// mtr_common.cuh -- numerics and helpers shared by the kernels of the fused
// decode-sampling step (mtr_sampler.cu: row-per-CTA and row-per-warp kernels;
// mtr_stream.cu: streaming row-group kernel).  Every decision-relevant
// operation lives here once, so all kernels are bit-identical to each other and
// to the CPU oracle.
#pragma once

#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/mtr_sampler.h"

namespace cg = cooperative_groups;

namespace mtr {

constexpr int NB = 1024;            // distance bins per histogram
constexpr float BIN_SCALE = 32.0f;  // bins per logit unit (d in [0, 32) before the overflow bin)
constexpr int CAP = 256;            // candidate list capacity
constexpr int MINI = 64;            // crossing-bin list capacity
constexpr int32_t NO_ID = 0x7fffffff;
constexpr unsigned FULL = 0xffffffffu;

typedef unsigned long long u64;

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }
__device__ __forceinline__ float pos_inf() { return __int_as_float(0x7f800000); }

// ---------------------------------------------------------------------------
// packed f32x2 arithmetic (sm_100a); each lane is one IEEE round-to-nearest op.
// Only fma / mul chains are used: they were checked bit-identical to the scalar
// sequence over every d in the exponential's range and 8M quotients.  ptxas
// rewrites packed mul -> add chains, so those stay scalar.
// ---------------------------------------------------------------------------
__device__ __forceinline__ u64 pk2(float a, float b) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(u64 r, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r)); }
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

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

// expfx on two values at once (same operations, packed); d0, d1 <= 0
__device__ __forceinline__ void expfx2(float d0, float d1, uint32_t& q0, uint32_t& q1) {
  const u64 D = pk2(d0, d1);
  float t0, t1;
  up2(mul2(D, pk2(0x1.715476p+0f, 0x1.715476p+0f)), t0, t1);
  const float n0 = rintf(t0), n1 = rintf(t1);
  const u64 Nn = pk2(n0, n1);
  u64 R = fma2(Nn, pk2(-0x1.62e400p-1f, -0x1.62e400p-1f), D);
  R = fma2(Nn, pk2(-0x1.7f7d1cp-20f, -0x1.7f7d1cp-20f), R);
  u64 P = pk2(0x1.6ab980p+21f, 0x1.6ab980p+21f);
  P = fma2(P, R, pk2(0x1.126d0cp+24f, 0x1.126d0cp+24f));
  P = fma2(P, R, pk2(0x1.55589ap+26f, 0x1.55589ap+26f));
  P = fma2(P, R, pk2(0x1.55540ap+28f, 0x1.55540ap+28f));
  P = fma2(P, R, pk2(0x1.fffffap+29f, 0x1.fffffap+29f));
  P = fma2(P, R, pk2(0x1.000000p+31f, 0x1.000000p+31f));
  P = fma2(P, R, pk2(0x1.000000p+31f, 0x1.000000p+31f));
  float p0, p1;
  up2(P, p0, p1);
  // |n| <= 46 whenever d >= -32; the clamp only keeps the shift defined
  const int s0 = -__float2int_rz(fmaxf(n0, -40.0f)), s1 = -__float2int_rz(fmaxf(n1, -40.0f));
  const uint32_t m0 = __float2uint_rz(p0), m1 = __float2uint_rz(p1);
  q0 = (d0 >= -32.0f && s0 < 32) ? (m0 >> s0) : 0u;
  q1 = (d1 >= -32.0f && s1 < 32) ? (m1 >> s1) : 0u;
}

// Natural logarithm in double precision, written for this project from the
// series ln x = e ln2 + 2 atanh(z), z = (f - 1) / (f + 1), x = f 2^e with f in
// [sqrt(1/2), sqrt(2)) (|z| <= 0.172, so twelve odd terms reach 2^-60).  Every
// step is a single IEEE-rounded double operation, so the CPU oracle's copy
// (compiled without contraction) gives the same bits.  Used by the lookback
// bias only, a few times per row.
__device__ __forceinline__ double log_d(double x) {
  if (x != x) return x;
  if (x < 0.0) return __longlong_as_double(0x7ff8000000000000LL);
  if (x == 0.0) return __longlong_as_double((long long)0xfff0000000000000ULL);
  if (x == __longlong_as_double(0x7ff0000000000000LL)) return x;
  int e = 0;
  unsigned long long b = (unsigned long long)__double_as_longlong(x);
  if ((b >> 52) == 0ull) {  // subnormal
    x = __dmul_rn(x, 0x1p54);
    b = (unsigned long long)__double_as_longlong(x);
    e = -54;
  }
  e += (int)(b >> 52) - 1023;
  double f = __longlong_as_double((long long)((b & 0x000fffffffffffffull) | 0x3ff0000000000000ull));
  if (f > 0x1.6a09e667f3bcdp+0) {
    f = __dmul_rn(f, 0.5);
    e += 1;
  }
  const double z = __ddiv_rn(__dsub_rn(f, 1.0), __dadd_rn(f, 1.0));
  const double w = __dmul_rn(z, z);
  double p = 0x1.642c8590b2164p-5;  // 1/23
  p = __dadd_rn(__dmul_rn(p, w), 0x1.8618618618618p-5);  // 1/21
  p = __dadd_rn(__dmul_rn(p, w), 0x1.af286bca1af28p-5);  // 1/19
  p = __dadd_rn(__dmul_rn(p, w), 0x1.e1e1e1e1e1e1ep-5);  // 1/17
  p = __dadd_rn(__dmul_rn(p, w), 0x1.1111111111111p-4);  // 1/15
  p = __dadd_rn(__dmul_rn(p, w), 0x1.3b13b13b13b14p-4);  // 1/13
  p = __dadd_rn(__dmul_rn(p, w), 0x1.745d1745d1746p-4);  // 1/11
  p = __dadd_rn(__dmul_rn(p, w), 0x1.c71c71c71c71cp-4);  // 1/9
  p = __dadd_rn(__dmul_rn(p, w), 0x1.2492492492492p-3);  // 1/7
  p = __dadd_rn(__dmul_rn(p, w), 0x1.999999999999ap-3);  // 1/5
  p = __dadd_rn(__dmul_rn(p, w), 0x1.5555555555555p-2);  // 1/3
  p = __dadd_rn(__dmul_rn(p, w), 1.0);
  return __dadd_rn(__dmul_rn((double)e, 0x1.62e42fefa39efp-1), __dmul_rn(__dmul_rn(2.0, z), p));
}

// The lookback bias's row constants (osuT5/osuT5/inference/logit_processors.py:150-166)
// from the fixed-point masses of the row before the bias: Q over every finite
// score, O over the ids outside [lb_start, lb_end), the previous step's EOS
// probability p.  s = 1 / ((O/Q)(1 - p) + p); the scores outside the range
// become x - c with c = max + ln(Q 2^-31) - ln s (the log of the renormalised
// probability), lb_start becomes ln(clip((s - 1) p / (1 - p), 0, 1)).
__device__ __forceinline__ void lookback_consts(u64 Q, u64 O, float pf, float mx, double* c, float* lbv) {
  const double p = (double)pf, pe = __dsub_rn(1.0, p);
  const double ratio = __ddiv_rn((double)O, (double)Q);
  const double s = __ddiv_rn(1.0, __dadd_rn(__dmul_rn(ratio, pe), p));
  double ex = __ddiv_rn(__dmul_rn(__dsub_rn(s, 1.0), p), pe);
  if (ex < 0.0) ex = 0.0;
  else if (ex > 1.0) ex = 1.0;
  const double lq = __dsub_rn(log_d((double)Q), __dmul_rn(31.0, 0x1.62e42fefa39efp-1));
  *c = __dsub_rn(__dadd_rn((double)mx, lq), log_d(s));
  *lbv = __double2float_rn(log_d(ex));
}

// x / t correctly rounded, given y = RN(1/t) (Markstein: q0 = x*y, r = x - q0*t
// exactly, q = q0 + r*y).  Magnitudes outside [2^-60, 2^60) and NaN take the
// IEEE divide; zeros and infinities pass through (t is positive and finite).
// out of line: the rare operands keep the IEEE divide away from the hot code
static __device__ __noinline__ float div_rare(float x, float t) {
  if (x == 0.0f || fabsf(x) == pos_inf()) return x;
  return __fdiv_rn(x, t);
}
__device__ __forceinline__ float div_by(float x, float t, float y) {
  const float ax = fabsf(x);
  if (ax >= 0x1p-60f && ax < 0x1p60f) {
    const float q0 = __fmul_rn(x, y);
    const float r = __fmaf_rn(-q0, t, x);
    return __fmaf_rn(r, y, q0);
  }
  return div_rare(x, t);
}

// the same on a pair; fma(q0, -t, x) is bit-identical to fma(-q0, t, x)
__device__ __forceinline__ void div_by2(float& x0, float& x1, float t, float y) {
  const u64 X = pk2(x0, x1), Y = pk2(y, y);
  const u64 Q0 = mul2(X, Y);
  const u64 Rr = fma2(Q0, pk2(-t, -t), X);
  float q0, q1;
  up2(fma2(Rr, Y, Q0), q0, q1);
  const float a0 = fabsf(x0), a1 = fabsf(x1);
  const bool ok0 = a0 >= 0x1p-60f && a0 < 0x1p60f, ok1 = a1 >= 0x1p-60f && a1 < 0x1p60f;
  const bool pass0 = x0 == 0.0f || a0 == pos_inf(), pass1 = x1 == 0.0f || a1 == pos_inf();
  if ((!ok0 && !pass0) || (!ok1 && !pass1)) {  // tiny, huge or NaN: rare
    q0 = ok0 || pass0 ? q0 : __fdiv_rn(x0, t);
    q1 = ok1 || pass1 ? q1 : __fdiv_rn(x1, t);
  }
  x0 = ok0 ? q0 : (pass0 ? x0 : q0);
  x1 = ok1 ? q1 : (pass1 ? x1 : q1);
}

// maxima that return NaN when any input is NaN (three-input form: sm_100)
__device__ __forceinline__ float fmax3n(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fmax2n(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

static __device__ __noinline__ void div_chunk_rare(float (&v)[8], float t, float y) {
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = div_by(v[e], t, y);
}

// x / t for a chunk (y = RN(1/t)): Markstein on pairs when every value that is
// not -inf lies in [2^-60, 2^60) (-inf passes through), the IEEE divide per
// element otherwise.
__device__ __forceinline__ void div_chunk(float (&v)[8], float t, float y) {
  float w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) w[e] = v[e] == neg_inf() ? 1.0f : fabsf(v[e]);
  const float amax = fmax3n(fmax3n(w[0], w[1], w[2]), fmax3n(w[3], w[4], w[5]), fmax2n(w[6], w[7]));
  const float amin = fminf(fminf(fminf(w[0], w[1]), fminf(w[2], w[3])), fminf(fminf(w[4], w[5]), fminf(w[6], w[7])));
  if (amax < 0x1p60f && amin >= 0x1p-60f) {
    const u64 Y = pk2(y, y), NT = pk2(-t, -t);
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const u64 Xv = pk2(v[e], v[e + 1]);
      const u64 Q0 = mul2(Xv, Y);
      float q0, q1;
      up2(fma2(fma2(Q0, NT, Xv), Y, Q0), q0, q1);
      v[e] = v[e] == neg_inf() ? v[e] : q0;
      v[e + 1] = v[e + 1] == neg_inf() ? v[e + 1] : q1;
    }
  } else {
    div_chunk_rare(v, t, y);
  }
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

// distance bin of a finite x below the row maximum mx (non-increasing in x).
// bin(x) <= b  <=>  (mx - x) < (b + 1) / BIN_SCALE for b < NB - 1 (the scaling
// by a power of two is exact).
__device__ __forceinline__ int dbin(float mx, float x) {
  float s = __fmul_rn(__fsub_rn(mx, x), BIN_SCALE);
  s = fminf(s, (float)(NB - 1));
  return __float2int_rz(s);
}

__device__ __forceinline__ bool finite_val(float x) { return fabsf(x) < pos_inf(); }

// Hint: pull [p, p + bytes) into L2 with one bulk prefetch (16-byte granules
// fully inside the range; nothing is read into the SM).
__device__ __forceinline__ void l2_prefetch(const void* p, size_t bytes) {
  const uintptr_t b0 = ((uintptr_t)p + 15u) & ~(uintptr_t)15u;
  const uintptr_t b1 = ((uintptr_t)p + bytes) & ~(uintptr_t)15u;
  if (b1 > b0 && b1 - b0 < (1u << 20))
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(b0), "r"((uint32_t)(b1 - b0)) : "memory");
}

// canonical order: higher score first, then lower token id
__device__ __forceinline__ bool canon_before(float xj, int32_t ij, float xi, int32_t ii) {
  return xj > xi || (xj == xi && ij < ii);
}

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
  // the 16-byte group starting at element i from scalar loads (ids >= V read as 0)
  __device__ static uint4 gather(const void* p, int i, int V) {
    const float* f = (const float*)p;
    uint4 r;
    r.x = i < V ? __float_as_uint(__ldcs(f + i)) : 0u;
    r.y = i + 1 < V ? __float_as_uint(__ldcs(f + i + 1)) : 0u;
    r.z = i + 2 < V ? __float_as_uint(__ldcs(f + i + 2)) : 0u;
    r.w = i + 3 < V ? __float_as_uint(__ldcs(f + i + 3)) : 0u;
    return r;
  }
};
// 16-bit types: the 16-byte group of 8 elements from scalar loads (ids >= V read as 0)
__device__ __forceinline__ uint4 gather_u16(const void* p, int i, int V) {
  const unsigned short* h = (const unsigned short*)p;
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t lo = i + 2 * k < V ? (uint32_t)__ldcs(h + i + 2 * k) : 0u;
    const uint32_t hi = i + 2 * k + 1 < V ? (uint32_t)__ldcs(h + i + 2 * k + 1) : 0u;
    w[k] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
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
  __device__ static uint4 gather(const void* p, int i, int V) { return gather_u16(p, i, V); }
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
  __device__ static uint4 gather(const void* p, int i, int V) { return gather_u16(p, i, V); }
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

// The end of a row's step, shared by every kernel (decode_loop.py:303-316):
// finished rows emit pad_id, EOS clears unfinished, the token is appended to
// the id buffer and the stop counters move.  Returns the emitted token; sets
// MTR_ROW_APPEND_SKIPPED in *status for an out-of-range id-buffer column.
__device__ __forceinline__ int64_t finish_token(const MtrSamplerArgs& a, int64_t row, int64_t tok, uint32_t* status) {
  bool live = true;
  if (a.unfinished) {
    live = a.unfinished[row] != 0;
    if (!live) tok = a.pad_id;
  }
  const bool eos = is_eos(a, tok);
  if (a.unfinished) a.unfinished[row] = (uint8_t)(live && !eos);
  if (a.stop_counts && live && eos) {
    atomicAdd(a.stop_counts, 1u);
    if (a.unfinished) atomicAdd(a.stop_counts + 1, 1u);
  }
  if (a.id_buffer) {
    const int32_t cur = a.cur_len_dev ? *a.cur_len_dev : a.cur_len;
    if (cur >= 0 && (int64_t)cur < a.id_buffer_row_stride) a.id_buffer[row * a.id_buffer_row_stride + cur] = tok;
    else *status |= MTR_ROW_APPEND_SKIPPED;
  }
  return tok;
}

// bits [lo, hi) of an 8-bit chunk mask (empty when hi <= lo)
__device__ __forceinline__ uint32_t range_bits(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 8);
  return hi > lo ? (((1u << hi) - 1u) & ~((1u << lo) - 1u)) : 0u;
}

// ---------------------------------------------------------------------------
// cluster helper: CS == 1 degenerates to the CTA
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// warp / block helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ u64 warp_sum_u64(u64 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
  return v;
}
__device__ __forceinline__ u64 warp_incl_scan_u64(u64 v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const u64 t = __shfl_up_sync(FULL, v, o);
    if (lane >= o) v += t;
  }
  return v;
}
__device__ __forceinline__ uint32_t warp_incl_scan_u32(uint32_t v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(FULL, v, o);
    if (lane >= o) v += t;
  }
  return v;
}


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
  int32_t id_shift;  // id >> id_shift < NB for every id < V
  int32_t gwords;    // 32-bit words per grammar vocabulary bitmap
  float temp_rcp;
  float cond_rcp[MTR_MAX_COND_TEMPS];
  float col_rcp[MTR_MAX_COL_TEMP_RANGES];
  // -1, -0 and 1 as launch parameters: FMAs with them stay FMAs (a compile-time
  // constant would let the compiler turn them into a mul + add pair and fuse it)
  float neg_one, neg_zero, one;
  float rep_rcp;  // RN(1 / repetition_penalty) when it lies in [2^-30, 2^30] (Markstein divide), else 0
  int32_t pdl;    // launched as a programmatic dependent (host-side launch choice)
};

// Warp bitonic sort of 32*E distinct (or zero) u64 keys, descending; lane l
// holds positions l*E .. l*E+E-1.

// Bitonic sort of 64 u64 keys held two per lane (positions 2*lane, 2*lane+1), descending.
__device__ __forceinline__ void sort64_desc(u64& a0, u64& a1, int lane) {
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j >= 2; j >>= 1) {
      const u64 p0 = __shfl_xor_sync(FULL, a0, j >> 1), p1 = __shfl_xor_sync(FULL, a1, j >> 1);
      const int g = 2 * lane;  // both positions share the bits k and j
      const bool keep_larger = ((g & k) == 0) == ((g & j) == 0);
      // keys are distinct except the empty (zero) entries, where taking either is the same
      if ((p0 > a0) == keep_larger) a0 = p0;
      if ((p1 > a1) == keep_larger) a1 = p1;
    }
    const bool desc = ((2 * lane) & k) == 0;
    const bool sw = (a0 < a1) == desc;
    const u64 t0 = sw ? a1 : a0, t1 = sw ? a0 : a1;
    a0 = t0;
    a1 = t1;
  }
}
// Bitonic sort of 128 u64 keys held four per lane (positions 4*lane .. 4*lane+3),
// descending; keys are distinct except the empty (zero) entries.  Stages whose
// partner lies in another lane exchange by shuffle, the last two of every block
// stay in registers.
__device__ __forceinline__ void sort128_desc(u64 (&v)[4], int lane) {
#pragma unroll
  for (int k = 2; k <= 128; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j >= 1; j >>= 1) {
      if (j >= 4) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const u64 p = __shfl_xor_sync(FULL, v[e], j >> 2);
          const int P = 4 * lane + e;
          const bool keep_larger = ((P & k) == 0) == ((P & j) == 0);
          if ((p > v[e]) == keep_larger) v[e] = p;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (e & j) continue;
          const bool desc = ((4 * lane + e) & k) == 0;  // the lower position keeps the larger key
          const u64 x = v[e], y = v[e | j];
          const bool sw = desc ? (x < y) : (x > y);
          v[e] = sw ? y : x;
          v[e | j] = sw ? x : y;
        }
      }
    }
  }
}
// repetition (x < 0 ? x * rp : x / rp), then frequency and presence, each step
// skipped when it is the identity (rp = 1, fp = 0, pp = 0); y = RN(1 / rp) or 0
__device__ __forceinline__ float pen_value(float x, float c, float rp, float fp, float pp, float y) {
  if (rp != 1.0f) x = x < 0.0f ? __fmul_rn(x, rp) : (y != 0.0f ? div_by(x, rp, y) : div_rare(x, rp));
  if (fp != 0.0f) x = __fsub_rn(x, __fmul_rn(fp, c));
  if (pp != 0.0f) x = __fsub_rn(x, pp);
  return x;
}

// Host side shared by the translation units of the library.
// Occupancy of a kernel at a launch shape, per device (computed once).
cudaError_t cached_occupancy(const void* kern, int threads, int dyn, int* occ);

// The streaming row-group kernel (mtr_stream.cu): whether it serves a request,
// its launch, and its launch shape for mtr_sampler_query_args.
bool sk_supported(const MtrSamplerArgs& a, const Derived& d);
cudaError_t stream_launch(const MtrSamplerArgs& a, const Derived& d, int sms, cudaStream_t s);
void stream_query(const MtrSamplerArgs& a, const Derived& d, int sms, MtrLaunchInfo* out);

// SM count of the current device (148 without a device), the thread's last CUDA
// error, and the sampler launch (validated arguments); `pdl` launches it as a
// programmatic dependent of the previous kernel on the stream (mtr_lmhead.cu).
int device_sms();
void set_last_cuda_error(int e);
int sampler_launch(const MtrSamplerArgs* a, cudaStream_t s, bool pdl);

// Launch attributes every sampler kernel launch shares: the cluster shape (when
// CS > 1) and programmatic stream serialisation (when d.pdl).
inline unsigned launch_attrs(cudaLaunchAttribute* at, int cs, bool pdl) {
  unsigned n = 0;
  if (cs > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = (unsigned)cs;
    at[n].val.clusterDim.y = 1;
    at[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  return n;
}

// Kernel entry of every sampler kernel: wait for the previous grid on the
// stream to complete with its memory visible (a no-op unless this launch is a
// programmatic dependent).
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Let the next programmatic dependent launch: its CTAs may be scheduled while
// this grid runs and wait at their own entry, so only launch latency overlaps,
// never data.  The row-per-CTA kernel calls it at entry; the persistent kernels
// do not (their early-finishing CTAs' slots would fill with waiting CTAs beside
// the last rows' warps), so their dependents launch as they exit.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace mtr
