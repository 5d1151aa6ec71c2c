// mtr_stream.cuh -- the streaming row-group kernel (throughput path of the fused
// decode-sampling step).  Device code only; it is instantiated per element type
// in mtr_stream_{bf16,f16,f32}.cu and launched from mtr_stream.cu.  It uses the
// shared numerics of mtr_common.cuh (expfx, Markstein division, packed f32x2
// FMAs, fkey, penalties) so its decisions are bit-identical to the other kernels
// and to the CPU oracle.
//
// A row group of G warps (G = 1, 2, 4, 8 or 16) owns one output row at a time
// and walks rows g, g + groups, ...  Nothing of the row is staged in shared
// memory: at the start of a row one thread issues bulk L2 prefetches of the
// row's logits and history window; thread t of the group then reads its 8-id
// chunks c = t, t + 32G, ... with 16-byte loads straight into registers (one
// chunk ahead) and keeps only the chunk maxima.  Shared memory per group is V bytes of history counts, V / 8
// bytes of history-presence bits and ~1.6 KB of lists, so 28 warps stay
// resident per SM at V = 4096.
//
//   history    the penalty window of input_ids -> u8 counts per id (shared
//              atomics; a row whose count of an id would pass 255 is counted
//              again with saturating updates and a small table of large counts)
//              and a presence bitmap; the monotonic full scan reads the same ids
//   pass 1     per chunk a keep byte (grammar bitmap of the previous token's
//              class, monotonic range, not a history id) is applied to the raw
//              16-bit words before CFG (first half -> -inf, second half -> 0, so
//              CFG yields exactly -inf); CFG as three packed FMAs
//              (second + (first - second) * scale); timeshift bias; chunk maximum
//   bound      64 bins of (row max - chunk max) * 8 (a second level at 1 logit
//              per bin when the first spills): with b* the first bin at which k
//              chunk maxima are reached, T = RD(max - (b* + 1) / 8) and at least
//              k elements (the maxima of k distinct chunks) score above T
//   listing    chunks whose maximum reaches T are read again (L2) and every
//              element >= T goes to the list as a canonical key
//              (score key << 32 | ~id); with a row temperature T is lowered by a
//              margin that covers the rounding of x / t
//   history    every distinct window id: score, masks, penalties from its count,
//              temperature, and a list entry when it reaches T.  When no penalty
//              can raise a score the unpenalised score filters first
//   selection  one warp: bitonic sort of <= 128 keys (canonical order), the k-th
//              key (ties kept), fixed-point masses q = floor(e^(x - max) 2^31),
//              top-p prefix of the exact 64-bit sums, draw through 32 id buckets
//   slow path  a list that overflows: the exact k-th value by radix select over
//              the row (read again), then the survivors listed, or -- when more
//              than 128 survivors tie at the k-th value -- the tie group kept as a
//              count whose lowest ids are taken, drawn by a walk in id order
//   outputs    processed scores / log-probs (optional) by one more walk
//
// Reference arithmetic: the same chain and decision rules as the row-per-CTA
// kernel (see the head of mtr_sampler.cu for the reference file:line list).
#pragma once

#include <stddef.h>

#include "mtr_common.cuh"

namespace mtr {

constexpr int SK_J = 16;                               // 8-id chunk slots per thread
constexpr int SK_MAX_G = 16;                           // warps per row group
constexpr int SK_MAX_VOCAB = 256 * SK_J * SK_MAX_G;    // 65536
constexpr int SK_CAP = 256;                            // candidate list per row
constexpr int SK_QCAP = 128;                           // qualifying-chunk list per row
constexpr int SK_TOPK_MAX = 64;                        // top-k served by this kernel
constexpr int SK_HEAVY = 16;                           // ids counted past 255 (8-bit counts)
constexpr int SK_HPT = 4;                              // history ids per thread and round (L2-prefetched)
constexpr int SK_LUT_BYTES = 128;                      // 16 keep-nibble -> 16-bit lane masks
constexpr uint32_t SK_EMPTY = 0xffffffffu;

// launch shapes: threads per CTA and the register budget that goes with them
enum SkShape { SK_SHAPE_128 = 0, SK_SHAPE_256 = 1, SK_SHAPE_512 = 2 };

// Host-derived geometry of one stream launch.
struct SkGeo {
  int32_t G;             // warps per row group
  int32_t R;             // row groups per CTA
  int32_t group_bytes;   // shared bytes per row group
  int32_t cnt_off;       // byte offset of the history counts inside a group's region
  int32_t pres_off;      // byte offset of the presence bitmap
  int32_t cnt16;         // 16-bit counts (windows of >= 256 * SK_HEAVY ids) instead of 8-bit + heavy table
  int32_t pen_fast;      // no penalty can raise a score (rep >= 1, freq >= 0, presence >= 0)
  int32_t bucket_shift;  // (V - 1) >> bucket_shift < 32
  float margin_abs;      // absolute part of the temperature margin on the listing bound
  // chunk bounds from packed 16-bit arithmetic (CFG rows of bf16 / f16 logits):
  // a = RN16(first * s16 + RN16(second * m16)) with s16 = RN16(scale), m16 =
  // RN16(1 - scale) is within kappa * |a| + lambda * |second| + bound_abs of
  // the exact fp32 CFG value
  int32_t bound_cfg;     // 1: use the packed bound (scale representable and > 0)
  uint32_t s16x2;        // s16 in both halves
  uint32_t m16x2;        // m16 in both halves
  float kappa, lambda, bound_abs;
};

struct SkLaunch {
  int threads, dyn, grid, shape;
  int j4;  // the 4-slot instantiation (4 * 256 * G >= V)
};

struct alignas(16) SkHead {
  uint32_t status;      // row status bits raised by single threads (OR into the group's)
  uint32_t nlist;       // list entries appended (can exceed SK_CAP: overflow)
  uint32_t nq;          // qualifying chunks (can exceed SK_QCAP)
  uint32_t ovf;         // an 8-bit count wrapped: count again with saturation
  int32_t bstar;
  int32_t token;
  uint32_t pad[2];
  u64 bc[6];            // selection results broadcast to the group
  uint32_t heavy_id[SK_HEAVY];
  uint32_t heavy_n[SK_HEAVY];
  u64 red[SK_MAX_G];    // cross-warp reductions
  uint32_t aux[64];     // bins / qualifying chunks (u16) / draw buckets
  u64 list[SK_CAP];     // canonical keys; the radix histogram (u32[256]) in the slow path
};

// per element type: 16-byte groups per 8-id chunk, the -inf pattern of a 32-bit
// word of raw elements, and the conversion of one word
template <typename T> struct SkT;
template <> struct SkT<__nv_bfloat16> {
  static constexpr int NV = 1;
  static constexpr uint32_t NEGW = 0xff80ff80u;
  __device__ static uint32_t pfma(uint32_t x, uint32_t y, uint32_t z) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(y), "r"(z));
    return d;
  }
  __device__ static uint32_t pmaxn(uint32_t x, uint32_t y) {
    uint32_t d;
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
    return d;
  }
  __device__ static void cvt(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  }
  __device__ static float one(const uint8_t* p, int i) {
    return __uint_as_float((uint32_t)__ldg((const unsigned short*)p + i) << 16);
  }
};
template <> struct SkT<__half> {
  static constexpr int NV = 1;
  static constexpr uint32_t NEGW = 0xfc00fc00u;
  __device__ static uint32_t pfma(uint32_t x, uint32_t y, uint32_t z) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(y), "r"(z));
    return d;
  }
  __device__ static uint32_t pmaxn(uint32_t x, uint32_t y) {
    uint32_t d;
    asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(x), "r"(y));
    return d;
  }
  __device__ static void cvt(uint32_t w, float& lo, float& hi) {
    lo = __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
    hi = __half2float(__ushort_as_half((unsigned short)(w >> 16)));
  }
  __device__ static float one(const uint8_t* p, int i) {
    return __half2float(__ushort_as_half(__ldg((const unsigned short*)p + i)));
  }
};
template <> struct SkT<float> {
  static constexpr int NV = 2;
  static constexpr uint32_t NEGW = 0xff800000u;
  __device__ static float one(const uint8_t* p, int i) { return __ldg((const float*)p + i); }
};

// streaming 16-byte load: no L1 allocation (each chunk is read once here; the
// listing pass reads the few it needs again from L2)
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ u64 sk_ckey(float x, int id) {
  return ((u64)fkey(x) << 32) | (u64)(uint32_t)(~(uint32_t)id);
}
__device__ __forceinline__ float sk_kval(u64 k) { return key2f((uint32_t)(k >> 32)); }
__device__ __forceinline__ int sk_kid(u64 k) { return (int)(~(uint32_t)k); }

__device__ __forceinline__ float sk_max8(const float (&y)[8]) {
  return fmax2n(fmax3n(y[0], y[1], y[2]), fmax3n(fmax3n(y[3], y[4], y[5]), y[6], y[7]));
}

// Bitonic sort of 32 * E u64 keys held E per lane (positions E*lane .. E*lane+E-1),
// descending.  Keys are distinct except zero padding.
template <int E>
__device__ __forceinline__ void sort_desc(u64 (&k)[E], int lane) {
#pragma unroll
  for (int kk = 2; kk <= 32 * E; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j >= 1; j >>= 1) {
      if (j >= E) {
#pragma unroll
        for (int i = 0; i < E; ++i) {
          const u64 p = __shfl_xor_sync(FULL, k[i], j / E);
          const int pos = E * lane + i;
          const bool desc = (pos & kk) == 0;
          const bool low = (pos & j) == 0;
          if ((p > k[i]) == (low == desc)) k[i] = p;
        }
      } else {
#pragma unroll
        for (int i = 0; i < E; ++i) {
          if (i & j) continue;
          const int i2 = i | j;
          const int pos = E * lane + i;
          const bool desc = (pos & kk) == 0;
          const bool sw = desc ? (k[i] < k[i2]) : (k[i] > k[i2]);
          const u64 t0 = sw ? k[i2] : k[i], t1 = sw ? k[i] : k[i2];
          k[i] = t0;
          k[i2] = t1;
        }
      }
    }
  }
}

// the CTA's dynamic shared memory: the keep-mask table, then one region per
// row group; every shared access is addressed from this symbol (offsets, not
// stored pointers), so the compiler emits shared-memory instructions
extern __shared__ __align__(16) uint8_t sk_smem[];

struct SkGroup {
  int G, GT, gt, lane, wig, bar;
  uint32_t red_off;  // byte offset of the group's reduction slots in sk_smem
  __device__ __forceinline__ u64* red() const { return (u64*)(sk_smem + red_off); }
  // named barriers 1..4 with immediate ids: a register id would make every
  // CTA reserve all 16 barriers and cap the CTAs resident per SM
  __device__ __forceinline__ void sync() const {
    if (G == 1) {
      __syncwarp();
    } else {
      switch (bar) {
        case 1: asm volatile("bar.sync 1, %0;" ::"r"(GT) : "memory"); break;
        case 2: asm volatile("bar.sync 2, %0;" ::"r"(GT) : "memory"); break;
        case 3: asm volatile("bar.sync 3, %0;" ::"r"(GT) : "memory"); break;
        default: asm volatile("bar.sync 4, %0;" ::"r"(GT) : "memory"); break;
      }
    }
  }
  __device__ __forceinline__ uint32_t max_u32(uint32_t v) const {
    v = __reduce_max_sync(FULL, v);
    if (G == 1) return v;
    if (lane == 0) red()[wig] = v;
    sync();
    uint32_t r = 0;
    for (int w = 0; w < G; ++w) r = max(r, (uint32_t)red()[w]);
    sync();
    return r;
  }
  __device__ __forceinline__ uint32_t or_u32(uint32_t v) const {
    v = __reduce_or_sync(FULL, v);
    if (G == 1) return v;
    if (lane == 0) red()[wig] = v;
    sync();
    uint32_t r = 0;
    for (int w = 0; w < G; ++w) r |= (uint32_t)red()[w];
    sync();
    return r;
  }
  __device__ __forceinline__ int max_i32(int v) const {
    v = __reduce_max_sync(FULL, v);
    if (G == 1) return v;
    if (lane == 0) red()[wig] = (u64)(uint32_t)v;
    sync();
    int r = INT32_MIN;
    for (int w = 0; w < G; ++w) r = max(r, (int)(uint32_t)red()[w]);
    sync();
    return r;
  }
  // inclusive scan in thread order (gt); *total = the group's sum
  __device__ __forceinline__ u64 scan_u64(u64 v, u64* total) const {
    u64 incl = warp_incl_scan_u64(v, lane);
    if (G == 1) {
      *total = __shfl_sync(FULL, incl, 31);
      return incl;
    }
    if (lane == 31) red()[wig] = incl;
    sync();
    u64 before = 0, tot = 0;
    for (int w = 0; w < G; ++w) {
      const u64 s = red()[w];
      if (w < wig) before += s;
      tot += s;
    }
    sync();
    *total = tot;
    return incl + before;
  }
};

// Per-row context.  In the hot path its fields live in registers; the rare
// paths (slow selection, output walk) are out of line and get a copy.
template <typename Tin, bool CFG>
struct SkRow {
  using T = SkT<Tin>;
  static constexpr int NV = T::NV;
  static constexpr int CB = 8 * (int)sizeof(Tin);  // bytes of one chunk and side

  const uint8_t* p1;  // first-half row
  const uint8_t* p2;  // partner row (CFG)
  const uint32_t* gb; // grammar bitmap of the previous token's class (null: no grammar mask)
  const uint8_t* idsr;  // this row of input_ids
  int64_t row;
  uint32_t goff;      // byte offset of the group's region in sk_smem
  uint32_t cnt_off;   // counts, relative to the region
  uint32_t pres_off;  // presence bitmap, relative to the region
  int V, nch, L, mono_lo, mono_hi, k_top;
  float t_row, t_rcp, u;
  bool pen_on, bias_on, cnt16;
  u64 NEG1, SC, NZ, ONE;
  SkGroup g;

  __device__ __forceinline__ SkHead& head() const { return *(SkHead*)(sk_smem + goff); }
  __device__ __forceinline__ uint32_t* cnt() const { return (uint32_t*)(sk_smem + goff + cnt_off); }
  __device__ __forceinline__ uint32_t* pres() const { return (uint32_t*)(sk_smem + goff + pres_off); }
  __device__ __forceinline__ const uint2* lut() const { return (const uint2*)sk_smem; }

  __device__ __forceinline__ void ld_chunk(int c, uint4 (&ra)[NV], uint4 (&rb)[NV]) const {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      ra[v] = ldg_stream(p1 + (size_t)c * CB + 16 * v);
      if constexpr (CFG) rb[v] = ldg_stream(p2 + (size_t)c * CB + 16 * v);
    }
  }
  __device__ __forceinline__ void ld_chunk_l2(int c, uint4 (&ra)[NV], uint4 (&rb)[NV]) const {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      ra[v] = __ldg((const uint4*)(p1 + (size_t)c * CB) + v);
      if constexpr (CFG) rb[v] = __ldg((const uint4*)(p2 + (size_t)c * CB) + v);
    }
  }
  __device__ __forceinline__ int64_t raw_id(const MtrSamplerArgs& a, int pos) const {
    if (a.ids_dtype == MTR_IDS_I32) return (int64_t)__ldg((const int32_t*)idsr + pos);
    return (int64_t)__ldg((const long long*)idsr + pos);
  }
  // low 32 bits of the id at pos, and (ok) whether it is a vocabulary id 0 <= id < V
  __device__ __forceinline__ uint32_t id_at(const MtrSamplerArgs& a, int pos, bool& ok) const {
    if (a.ids_dtype == MTR_IDS_I32) {
      const uint32_t t = (uint32_t)__ldg((const int32_t*)idsr + pos);
      ok = t < (uint32_t)V;
      return t;
    }
    const uint2 w = __ldg((const uint2*)idsr + pos);
    ok = w.y == 0u && w.x < (uint32_t)V;
    return w.x;
  }
  // penalty count of id t (0 <= t < V)
  __device__ __forceinline__ uint32_t count_of(int t) const {
    if (cnt16) return (cnt()[t >> 1] >> (16 * (t & 1))) & 0xffffu;
    uint32_t c = (cnt()[t >> 2] >> (8 * (t & 3))) & 0xffu;
    if (c == 255u) {
      const SkHead& h = head();
#pragma unroll 1
      for (int i = 0; i < SK_HEAVY; ++i)
        if (h.heavy_id[i] == (uint32_t)t) c += h.heavy_n[i];
    }
    return c;
  }
  // keep byte of chunk c: grammar, monotonic range and (excl_hist) not a history id
  __device__ __forceinline__ uint32_t keep_of(int c, bool excl_hist) const {
    uint32_t keep = 0xffu;
    if (gb) keep = __ldg(gb + (c >> 2)) >> (8 * (c & 3));
    if (excl_hist && pen_on) keep &= ~(pres()[c >> 2] >> (8 * (c & 3)));
    keep &= ~range_bits(mono_lo - 8 * c, mono_hi - 8 * c);
    return keep & 0xffu;
  }
  __device__ __forceinline__ void add_bias(const MtrSamplerArgs& a, float (&y)[8], int id0) const {
    if (id0 + 8 <= a.ts_start || id0 >= a.ts_end) return;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (id0 + e >= a.ts_start && id0 + e < a.ts_end) y[e] = __fadd_rn(y[e], a.timeshift_bias);
  }
  // Masked, CFG-combined values of one chunk.  Keep bit e = element e survives
  // the masks; a masked first-half element becomes -inf and its partner 0 before
  // CFG, which then yields exactly -inf whatever the raw values were.
  __device__ __forceinline__ void chunk_y(const uint4 (&A)[NV], const uint4 (&B)[NV], uint32_t keep,
                                          float (&y)[8]) const {
    const uint2 m01 = lut()[keep & 15u], m23 = lut()[(keep >> 4) & 15u];
    const uint32_t mw[4] = {m01.x, m01.y, m23.x, m23.y};
    if constexpr (sizeof(Tin) == 2) {
      const uint32_t wa[4] = {A[0].x, A[0].y, A[0].z, A[0].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t ca = (wa[i] & mw[i]) | (~mw[i] & T::NEGW);
        float f0, f1;
        T::cvt(ca, f0, f1);
        if constexpr (CFG) {
          const uint32_t wb[4] = {B[0].x, B[0].y, B[0].z, B[0].w};
          float g0, g1;
          T::cvt(wb[i] & mw[i], g0, g1);
          const u64 Q = pk2(g0, g1);
          u64 D = fma2(Q, NEG1, pk2(f0, f1));  // first - second
          D = fma2(D, SC, NZ);                  // * scale
          D = fma2(D, ONE, Q);                  // + second
          up2(D, y[2 * i], y[2 * i + 1]);
        } else {
          y[2 * i] = f0;
          y[2 * i + 1] = f1;
        }
      }
    } else {
      const uint32_t wa[8] = {A[0].x, A[0].y, A[0].z, A[0].w, A[1].x, A[1].y, A[1].z, A[1].w};
      float f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t m = __byte_perm(mw[e >> 1], 0u, (e & 1) ? 0x2222u : 0x0000u);
        f[e] = __uint_as_float((wa[e] & m) | (~m & T::NEGW));
      }
      if constexpr (CFG) {
        const uint32_t wb[8] = {B[0].x, B[0].y, B[0].z, B[0].w, B[1].x, B[1].y, B[1].z, B[1].w};
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint32_t m0 = __byte_perm(mw[e >> 1], 0u, 0x0000u), m1 = __byte_perm(mw[e >> 1], 0u, 0x2222u);
          const u64 Q = pk2(__uint_as_float(wb[e] & m0), __uint_as_float(wb[e + 1] & m1));
          u64 D = fma2(Q, NEG1, pk2(f[e], f[e + 1]));
          D = fma2(D, SC, NZ);
          D = fma2(D, ONE, Q);
          up2(D, y[e], y[e + 1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = f[e];
      }
    }
  }
  // Bounds of the masked chunk (16-bit types): amax = the largest masked
  // first-half element (no CFG) or the largest packed approximation a (CFG),
  // NaN when any is NaN; umax = the largest |second-half element| (CFG).
  __device__ __forceinline__ void chunk_bound(const uint4 (&A)[NV], const uint4 (&B)[NV], uint32_t keep, uint32_t s2,
                                              uint32_t m2, float& amax, float& umax) const {
    if constexpr (sizeof(Tin) == 2) {
      const uint2 m01 = lut()[keep & 15u], m23 = lut()[(keep >> 4) & 15u];
      const uint32_t mw[4] = {m01.x, m01.y, m23.x, m23.y};
      const uint32_t wa[4] = {A[0].x, A[0].y, A[0].z, A[0].w};
      uint32_t am = 0, um = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t w = (wa[i] & mw[i]) | (~mw[i] & T::NEGW);
        if constexpr (CFG) {
          const uint32_t wb[4] = {B[0].x, B[0].y, B[0].z, B[0].w};
          const uint32_t ub = wb[i] & mw[i];
          w = T::pfma(w, s2, T::pfma(ub, m2, 0u));
          const uint32_t ua = ub & 0x7fff7fffu;
          um = i ? T::pmaxn(um, ua) : ua;
        }
        am = i ? T::pmaxn(am, w) : w;
      }
      float lo, hi;
      T::cvt(am, lo, hi);
      amax = fmax2n(lo, hi);
      if constexpr (CFG) {
        T::cvt(um, lo, hi);
        umax = fmax2n(lo, hi);
      } else {
        umax = 0.0f;
      }
    } else {
      amax = neg_inf();
      umax = 0.0f;
    }
  }
  // final scores of chunk c (every step of the chain; history ids penalised from
  // their counts), read again from L2
  __device__ __forceinline__ void full_chunk(const MtrSamplerArgs& a, const Derived& dv, int c, float (&x)[8]) const {
    uint4 ra[NV], rb[NV];
    ld_chunk_l2(c, ra, rb);
    chunk_y(ra, rb, keep_of(c, false), x);
    if (bias_on) add_bias(a, x, 8 * c);
    if (pen_on) {
      const float rp = a.repetition_penalty, fp = a.frequency_penalty, pp = a.presence_penalty;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t n = count_of(8 * c + e);
        if (n) x[e] = pen_value(x[e], (float)n, rp, fp, pp, dv.rep_rcp);
      }
    }
    if (t_row != 1.0f) div_chunk(x, t_row, t_rcp);
  }
  // score of one id before penalties and temperature (masks, CFG, bias)
  __device__ __forceinline__ float elem_y(const MtrSamplerArgs& a, const Derived& dv, int t) const {
    const bool masked = (gb && !((__ldg(gb + (t >> 5)) >> (t & 31)) & 1u)) || (t >= mono_lo && t < mono_hi);
    if (masked) return neg_inf();
    float y;
    const float c1 = T::one(p1, t);
    if constexpr (CFG) {
      const float c2 = T::one(p2, t);
      const float d = __fmaf_rn(c2, dv.neg_one, c1);
      const float m = __fmaf_rn(d, a.cfg_scale, dv.neg_zero);
      y = __fmaf_rn(m, dv.one, c2);
    } else {
      y = c1;
    }
    if (bias_on && t >= a.ts_start && t < a.ts_end) y = __fadd_rn(y, a.timeshift_bias);
    return y;
  }
  // list append: every lane of the warp calls; bit e of sel lists x[e] with
  // id id0 + e (ids == nullptr) or ids[e]
  template <int N>
  __device__ __forceinline__ void append(uint32_t sel, const float (&x)[N], int id0, const int* ids = nullptr) const {
    if (!__any_sync(FULL, sel != 0u)) return;
    const uint32_t n = __popc(sel);
    const uint32_t incl = warp_incl_scan_u32(n, g.lane);
    const uint32_t tot = __shfl_sync(FULL, incl, 31);
    SkHead& h = head();
    uint32_t base = 0;
    if (g.lane == 31) base = atomicAdd(&h.nlist, tot);
    base = __shfl_sync(FULL, base, 31);
    uint32_t s = base + incl - n;
#pragma unroll
    for (int e = 0; e < N; ++e) {
      if ((sel >> e) & 1u) {
        if (s < (uint32_t)SK_CAP) h.list[s] = sk_ckey(x[e], ids ? ids[e] : id0 + e);
        ++s;
      }
    }
  }
};

// Selection results of a row (written by the selecting warp, read by the group).
//   mode 0: the kept set is every canonical key >= kcut
//   mode 1: tie mode -- kept = strict keys >= kcut (kcut = 0: none) plus the
//           nstar lowest ids scoring exactly key2f(kth)
struct SkSel {
  u64 kcut;
  u64 qkept;
  u64 target;
  float mx;
  uint32_t kth;
  uint32_t nstar;
  int mode;
  int token;
};

// One warp: sort the list (n <= SK_CAP keys at h->list), top-k, top-p, draw.
// Results go to h->token / h->bc[0..2]; the row-level status bit to h->status.
template <int E, typename Tin, bool CFG>
__device__ __forceinline__ void sk_select_e(const SkRow<Tin, CFG>& r, const MtrSamplerArgs& a, int bucket_shift, int n,
                                            bool sample, bool topp_on) {
  const int lane = r.g.lane;
  SkHead& h = r.head();
  u64 key[E];
#pragma unroll
  for (int i = 0; i < E; ++i) key[i] = E * lane + i < n ? h.list[E * lane + i] : 0ull;
  sort_desc<E>(key, lane);
  // the key at canonical position p (every lane gets it)
  auto key_at = [&](int p) __attribute__((always_inline)) -> u64 {
    u64 v = key[0];
#pragma unroll
    for (int i = 1; i < E; ++i)
      if ((p & (E - 1)) == i) v = key[i];
    return __shfl_sync(FULL, v, p / E);
  };
  // k-th key (ties kept): survivors are the keys whose score key reaches it
  uint32_t kv = 0;  // score keys are > 0 for finite scores
  if (n >= r.k_top) kv = (uint32_t)(key_at(r.k_top - 1) >> 32);
  const float M = sk_kval(__shfl_sync(FULL, key[0], 0));
  uint32_t q[E];
  bool surv[E];
#pragma unroll
  for (int i = 0; i < E; ++i) surv[i] = key[i] != 0ull && (uint32_t)(key[i] >> 32) >= kv;
#pragma unroll
  for (int i = 0; i < E; i += 2)
    expfx2(surv[i] ? __fsub_rn(sk_kval(key[i]), M) : -64.0f, surv[i + 1] ? __fsub_rn(sk_kval(key[i + 1]), M) : -64.0f,
           q[i], q[i + 1]);
  u64 lsum = 0;
#pragma unroll
  for (int i = 0; i < E; ++i) {
    if (!surv[i]) q[i] = 0u;
    lsum += q[i];
  }
  bool kept[E];
#pragma unroll
  for (int i = 0; i < E; ++i) kept[i] = surv[i];
  if (topp_on) {
    const u64 incl = warp_incl_scan_u64(lsum, lane);
    const u64 Q = __shfl_sync(FULL, incl, 31);
    const double P = __dmul_rn((double)a.top_p, (double)Q);
    const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
    u64 above = incl - lsum;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      kept[i] = surv[i] && above <= plim;
      above += q[i];
    }
  }
  // kept is a prefix of the canonical order: its length and last key
  uint32_t nk = 0, ns = 0;
#pragma unroll
  for (int i = 0; i < E; ++i) {
    nk += __popc(__ballot_sync(FULL, kept[i]));
    ns += __popc(__ballot_sync(FULL, surv[i]));
  }
  const u64 last = key_at((int)nk - 1);
  bool tie = false;
  if (topp_on && nk < ns) tie = (uint32_t)(key_at((int)nk) >> 32) == (uint32_t)(last >> 32);
  u64 ksum = 0;
#pragma unroll
  for (int i = 0; i < E; ++i)
    if (kept[i]) ksum += q[i];
  const u64 QK = warp_sum_u64(ksum);
  int tok = -1;
  if (sample) {
    const u64 tg = __double2ull_rz(floor(__dmul_rn((double)r.u, (double)QK)));
    // 32 id buckets of the kept mass (low / high 16 bits apart: 32-bit atomics)
    uint32_t* blo = h.aux;
    uint32_t* bhi = h.aux + 32;
    blo[lane] = 0u;
    bhi[lane] = 0u;
    __syncwarp();
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if (kept[i]) {
        const int b = sk_kid(key[i]) >> bucket_shift;
        atomicAdd(blo + b, q[i] & 0xffffu);
        atomicAdd(bhi + b, q[i] >> 16);
      }
    }
    __syncwarp();
    const u64 s = (u64)blo[lane] + ((u64)bhi[lane] << 16);
    const u64 incl = warp_incl_scan_u64(s, lane);
    const unsigned bal = __ballot_sync(FULL, incl - s <= tg && tg < incl);
    const int bb = __ffs(bal) - 1;  // exists: tg < QK
    u64 acc = __shfl_sync(FULL, incl - s, bb);
    bool mem[E];
#pragma unroll
    for (int i = 0; i < E; ++i) mem[i] = kept[i] && (sk_kid(key[i]) >> bucket_shift) == bb;
    // the bucket's kept ids in ascending order until the prefix passes the target
#pragma unroll 1
    for (int it = 0; it < 32 * E; ++it) {
      uint32_t mine = 0xffffffffu;
#pragma unroll
      for (int i = 0; i < E; ++i)
        if (mem[i]) mine = min(mine, (uint32_t)sk_kid(key[i]));
      const uint32_t mid = __reduce_min_sync(FULL, mine);
      if (mid == 0xffffffffu) break;
      uint32_t qm = 0;
#pragma unroll
      for (int i = 0; i < E; ++i)
        if (mem[i] && (uint32_t)sk_kid(key[i]) == mid) {
          qm = q[i];
          mem[i] = false;
        }
      acc += (u64)__reduce_add_sync(FULL, qm);
      if (acc > tg) {
        tok = (int)mid;
        break;
      }
    }
  }
  if (lane == 0) {
    h.token = tok;
    h.bc[0] = last;
    h.bc[1] = (u64)__float_as_uint(M);
    h.bc[2] = QK;
    if (tie) atomicOr(&h.status, MTR_ROW_TIE_AT_CUT);
  }
}

// One warp: the list of n <= SK_CAP keys sorted in registers (2, 4 or 8 per lane).
template <typename Tin, bool CFG>
__device__ __forceinline__ void sk_select_list(const SkRow<Tin, CFG>& r, const MtrSamplerArgs& a, int bucket_shift, int n,
                                               bool sample, bool topp_on) {
  if (n <= 64) sk_select_e<2>(r, a, bucket_shift, n, sample, topp_on);
  else if (n <= 128) sk_select_e<4>(r, a, bucket_shift, n, sample, topp_on);
  else sk_select_e<8>(r, a, bucket_shift, n, sample, topp_on);
}

// Slow selection (out of line): the list overflowed, or the test hook forces
// it.  Exact k-th score key by radix select over the row (read again), then
// either the survivors listed and selected as usual, or the tie mode.  Every
// thread of the group calls; the results come back in *out.
template <typename Tin, bool CFG>
__device__ __noinline__ void sk_slow_select(const SkRow<Tin, CFG> r, const MtrSamplerArgs& a, const Derived& dv,
                                            int bucket_shift, bool sample, bool topp_on, SkSel* out) {
  const SkGroup& g = r.g;
  SkHead& h = r.head();
  const int gt = g.gt, GT = g.GT, lane = g.lane;
  const float NEG = neg_inf();
  uint32_t* hist = (uint32_t*)h.list;
  uint32_t prefix = 0, rank = (uint32_t)r.k_top, n_gt = 0, n_eq = 0, nfin = 0;
  bool topk = true;
#pragma unroll 1
  for (int p = 0; p < 4; ++p) {
    const int sh = 24 - 8 * p;
    for (int i = gt; i < 256; i += GT) hist[i] = 0u;
    g.sync();
#pragma unroll 1
    for (int j = 0; j < SK_J; ++j) {
      const int c = j * GT + gt;
      if (c >= r.nch) continue;
      float x[8];
      r.full_chunk(a, dv, c, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (!(x[e] > NEG)) continue;
        const uint32_t kx = fkey(x[e]);
        if (p == 0 || (kx >> (sh + 8)) == prefix) atomicAdd(hist + ((kx >> sh) & 255u), 1u);
      }
    }
    g.sync();
    if (g.wig == 0) {
      // lane l owns digits 255 - 8l .. 248 - 8l (descending)
      uint32_t v[8], s = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        v[q] = hist[255 - 8 * lane - q];
        s += v[q];
      }
      const uint32_t incl = warp_incl_scan_u32(s, lane);
      const uint32_t tot = __shfl_sync(FULL, incl, 31);
      int dig = -1;
      uint32_t above = 0, w = 0;
      if (incl - s < rank && rank <= incl) {
        uint32_t c = incl - s;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (dig < 0 && c + v[q] >= rank) {
            dig = 255 - 8 * lane - q;
            above = c;
            w = v[q];
          }
          c += v[q];
        }
      }
      // the crossing digit (none only when rank > tot: the row has <= k finite scores)
      const unsigned bal = __ballot_sync(FULL, dig >= 0);
      const int src = bal ? __ffs(bal) - 1 : 0;
      const int d2 = __shfl_sync(FULL, dig, src);
      const uint32_t ab2 = __shfl_sync(FULL, above, src);
      const uint32_t w2 = __shfl_sync(FULL, w, src);
      if (lane == 0) {
        h.bc[3] = (u64)tot;
        h.bc[4] = (u64)(uint32_t)d2;
        h.bc[5] = ((u64)ab2 << 32) | w2;
      }
    }
    g.sync();
    const uint32_t tot = (uint32_t)h.bc[3];
    const int dig = (int)(uint32_t)h.bc[4];
    const uint32_t above = (uint32_t)(h.bc[5] >> 32), w = (uint32_t)h.bc[5];
    g.sync();
    if (p == 0) {
      nfin = tot;
      if (nfin <= (uint32_t)r.k_top) {
        topk = false;
        break;
      }
    }
    prefix = (prefix << 8) | (uint32_t)dig;
    rank -= above;
    n_gt += above;
    if (p == 3) n_eq = w;
  }
  const uint32_t ns = topk ? n_gt + n_eq : nfin;
  // list the survivors (or, with a tie group past the list, the strict ones)
  const bool ties = topk && ns > (uint32_t)SK_CAP;
  if (gt == 0) h.nlist = 0u;
  g.sync();
#pragma unroll 1
  for (int j = 0; j < SK_J; ++j) {
    const int c = j * GT + gt;
    float x[8];
    uint32_t sel = 0;
    if (c < r.nch) {
      r.full_chunk(a, dv, c, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (!(x[e] > NEG)) continue;
        const uint32_t kx = fkey(x[e]);
        if (!topk || (ties ? kx > prefix : kx >= prefix)) sel |= 1u << e;
      }
    }
    r.append(sel, x, 8 * (c < r.nch ? c : 0));
  }
  g.sync();
  SkSel s;
  s.mode = 0;
  s.kth = 0;
  s.nstar = 0;
  s.target = 0;
  if (!ties) {
    if (g.wig == 0) sk_select_list(r, a, bucket_shift, (int)h.nlist, sample, topp_on);
    g.sync();
    s.token = h.token;
    s.kcut = h.bc[0];
    s.mx = __uint_as_float((uint32_t)h.bc[1]);
    s.qkept = h.bc[2];
    g.sync();
    *out = s;
    return;
  }
  // tie mode: strict keys in the list (< k of them), the tie group at key `prefix`
  if (g.wig == 0) {
    const int n = (int)h.nlist;
    u64 k0 = 2 * lane < n ? h.list[2 * lane] : 0ull, k1 = 2 * lane + 1 < n ? h.list[2 * lane + 1] : 0ull;
    sort64_desc(k0, k1, lane);
    const float tval = key2f(prefix);
    const float M = n > 0 ? sk_kval(__shfl_sync(FULL, k0, 0)) : tval;
    uint32_t q0, q1, qt, qdummy;
    expfx2(k0 ? __fsub_rn(sk_kval(k0), M) : -64.0f, k1 ? __fsub_rn(sk_kval(k1), M) : -64.0f, q0, q1);
    expfx2(__fsub_rn(tval, M), -64.0f, qt, qdummy);
    if (!k0) q0 = 0u;
    if (!k1) q1 = 0u;
    const u64 lsum = (u64)q0 + q1;
    const u64 incl = warp_incl_scan_u64(lsum, lane);
    const u64 Qs = __shfl_sync(FULL, incl, 31);
    const u64 Q = Qs + (u64)n_eq * qt;
    bool kp0 = k0 != 0ull, kp1 = k1 != 0ull;
    uint32_t ns_kept = (uint32_t)n, nst = n_eq;
    bool tie = false;
    if (topp_on) {
      const double P = __dmul_rn((double)a.top_p, (double)Q);
      const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
      const u64 a0 = incl - lsum, a1 = a0 + q0;
      kp0 = kp0 && a0 <= plim;
      kp1 = kp1 && a1 <= plim;
      ns_kept = __popc(__ballot_sync(FULL, kp0)) + __popc(__ballot_sync(FULL, kp1));
      if (ns_kept == (uint32_t)n && Qs <= plim)
        nst = qt == 0u ? n_eq : (uint32_t)min((u64)n_eq, (plim - Qs) / qt + 1ull);
      else
        nst = 0u;
      // canonical neighbours at the cut: inside the strict keys, or inside the tie group
      if (ns_kept < (uint32_t)n) {
        const int pl = (int)ns_kept - 1, pn = (int)ns_kept;
        const u64 kl = __shfl_sync(FULL, (pl & 1) ? k1 : k0, pl >> 1);
        const u64 kn = __shfl_sync(FULL, (pn & 1) ? k1 : k0, pn >> 1);
        tie = ns_kept > 0 && (uint32_t)(kl >> 32) == (uint32_t)(kn >> 32);
      } else {
        tie = nst > 0u && nst < n_eq;
      }
    }
    const u64 ksum = (kp0 ? (u64)q0 : 0ull) + (kp1 ? (u64)q1 : 0ull);
    const u64 QK = warp_sum_u64(ksum) + (u64)nst * qt;
    u64 lastk = 0;
    if (ns_kept > 0) {
      const int pl = (int)ns_kept - 1;
      lastk = __shfl_sync(FULL, (pl & 1) ? k1 : k0, pl >> 1);
    }
    if (lane == 0) {
      h.bc[0] = lastk;
      h.bc[1] = (u64)__float_as_uint(M);
      h.bc[2] = QK;
      h.bc[3] = (u64)nst;
      h.bc[4] = sample ? __double2ull_rz(floor(__dmul_rn((double)r.u, (double)QK))) : 0ull;
      if (tie) atomicOr(&h.status, MTR_ROW_TIE_AT_CUT);
    }
  }
  g.sync();
  s.mode = 1;
  s.kth = prefix;
  s.kcut = h.bc[0];
  s.mx = __uint_as_float((uint32_t)h.bc[1]);
  s.qkept = h.bc[2];
  s.nstar = (uint32_t)h.bc[3];
  s.target = h.bc[4];
  s.token = -1;
  g.sync();
  *out = s;
}

// Walk over the row in id order (out of line): processed scores / log-probs,
// and the draw of the tie mode.  sel_ok: the row was selected (clean, not all
// masked).  Returns the drawn token of the tie mode through h->token.
template <typename Tin, bool CFG>
__device__ __noinline__ void sk_walk(const SkRow<Tin, CFG> r, const MtrSamplerArgs& a, const Derived& dv, const SkSel s,
                                     bool sel_ok, bool draw_walk) {
  const SkGroup& g = r.g;
  SkHead& h = r.head();
  const int gt = g.gt, GT = g.GT;
  const float NEG = neg_inf();
  const bool want_out = a.out_scores != nullptr || a.out_logprobs != nullptr;
  const double lse = sel_ok ? log((double)s.qkept) - 31.0 * 0.69314718055994530942 : 0.0;
  u64 run_mass = 0;
  uint32_t run_ties = 0;
  bool found = false;
#pragma unroll 1
  for (int j = 0; j < SK_J; ++j) {
    if (j * GT >= r.nch) break;
    const int c = j * GT + gt;
    const bool valid = c < r.nch;
    float x[8];
    if (valid) {
      r.full_chunk(a, dv, c, x);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = NEG;
    }
    bool kept[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) kept[e] = false;
    if (sel_ok) {
      uint32_t tie_flags = 0;
      u64 tie_tot = 0;
      uint32_t tie_before = 0;
      if (s.mode == 1) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (x[e] > NEG && fkey(x[e]) == s.kth) tie_flags |= 1u << e;
        const uint32_t tie_n = __popc(tie_flags);
        tie_before = (uint32_t)(g.scan_u64(tie_n, &tie_tot) - tie_n) + run_ties;
      }
      uint32_t tie_local = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (!(x[e] > NEG)) continue;
        const u64 ck = sk_ckey(x[e], 8 * c + e);
        if (s.mode == 0) {
          kept[e] = ck >= s.kcut;
        } else if ((tie_flags >> e) & 1u) {
          kept[e] = tie_before + tie_local < s.nstar;
          ++tie_local;
        } else {
          kept[e] = s.kcut != 0ull && ck >= s.kcut && fkey(x[e]) > s.kth;
        }
      }
      run_ties += (uint32_t)tie_tot;
      if (draw_walk && !found) {
        uint32_t q[8];
        float d[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) d[e] = kept[e] ? __fsub_rn(x[e], s.mx) : -64.0f;
#pragma unroll
        for (int e = 0; e < 8; e += 2) expfx2(d[e], d[e + 1], q[e], q[e + 1]);
        u64 sum = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (!kept[e]) q[e] = 0u;
          sum += q[e];
        }
        u64 tot = 0;
        const u64 incl = g.scan_u64(sum, &tot);
        const u64 lo = run_mass + incl - sum;
        if (lo <= s.target && s.target < run_mass + incl) {
          u64 acc = lo;
          int tk = -1;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            acc += q[e];
            if (tk < 0 && kept[e] && acc > s.target) tk = 8 * c + e;
          }
          h.token = tk;
        }
        run_mass += tot;
        found = s.target < run_mass;
      }
    }
    if (valid && a.out_scores) {
      float* o = a.out_scores + r.row * a.out_scores_row_stride + 8 * c;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (sel_ok && !kept[e]) ? NEG : x[e];
    }
    if (valid && a.out_logprobs) {
      float* o = a.out_logprobs + r.row * a.out_logprobs_row_stride + 8 * c;
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e] = !sel_ok ? __int_as_float(0x7fc00000) : (kept[e] ? (float)(((double)x[e] - (double)s.mx) - lse) : NEG);
    }
    if (!want_out && found) break;
  }
  g.sync();
}

// J: 8-id chunk slots per thread (4 or SK_J); the host picks J = 4 when
// 4 * 256 * G >= V, so no slot array is sized beyond what the row needs.
template <typename Tin, bool CFG, int MAXT, int MINB, int J>
__global__ void __launch_bounds__(MAXT, MINB) stream_kernel(const __grid_constant__ MtrSamplerArgs a,
                                                          const __grid_constant__ Derived dv,
                                                          const __grid_constant__ SkGeo geo) {
  wait_prior_grid();
  using T = SkT<Tin>;
  constexpr int NV = T::NV;
  const int tid = threadIdx.x;
  SkRow<Tin, CFG> r;
  r.g.G = geo.G;
  r.g.GT = geo.G * 32;
  const int grp = tid / r.g.GT;
  r.g.gt = tid - grp * r.g.GT;
  r.g.lane = tid & 31;
  r.g.wig = r.g.gt >> 5;
  r.g.bar = 1 + grp;
  r.goff = (uint32_t)(SK_LUT_BYTES + grp * geo.group_bytes);
  r.g.red_off = r.goff + (uint32_t)offsetof(SkHead, red);
  r.cnt_off = (uint32_t)geo.cnt_off;
  r.pres_off = (uint32_t)geo.pres_off;
  r.cnt16 = geo.cnt16 != 0;
  r.V = a.vocab;
  r.nch = a.vocab >> 3;
  r.L = a.input_ids ? dv.ids_len : 0;
  r.k_top = a.top_k;
  r.pen_on = dv.pen_on != 0;
  r.bias_on = a.timeshift_bias != 0.0f;
  r.NEG1 = pk2(dv.neg_one, dv.neg_one);
  r.NZ = pk2(dv.neg_zero, dv.neg_zero);
  r.ONE = pk2(dv.one, dv.one);
  r.SC = pk2(a.cfg_scale, a.cfg_scale);
  const SkGroup& g = r.g;
  SkHead& h = r.head();
  uint32_t* const cnt = r.cnt();
  uint32_t* const pres = r.pres();
  const int gt = g.gt, GT = g.GT, lane = g.lane;
  const int V = r.V, nch = r.nch, L = r.L;
  const int cnt_words = geo.cnt16 ? (V + 1) / 2 : (V + 3) / 4;
  const int pres_words = (V + 31) / 32;
  const bool scan_mode = a.mono_mode == MTR_MONO_SCAN;
  const float NEG = neg_inf();
  const size_t row_bytes = (size_t)a.logits_row_stride * sizeof(Tin);
  const bool want_out = a.out_scores != nullptr || a.out_logprobs != nullptr;
  const bool topp_on = dv.topp_on != 0;
  const bool sample = a.select_mode == MTR_SELECT_SAMPLE;
  const size_t ids_esz = a.ids_dtype == MTR_IDS_I32 ? 4 : 8;

  if (tid < 16)
    ((uint2*)sk_smem)[tid] = make_uint2(((tid & 1) ? 0xffffu : 0u) | ((tid & 2) ? 0xffff0000u : 0u),
                                    ((tid & 4) ? 0xffffu : 0u) | ((tid & 8) ? 0xffff0000u : 0u));
  // this group's tables start empty; every row leaves them empty again
  auto clear_tables = [&]() __attribute__((always_inline)) {
    for (int w = gt * 4; w < cnt_words; w += GT * 4) *(uint4*)(cnt + w) = make_uint4(0u, 0u, 0u, 0u);
    for (int w = gt; w < pres_words; w += GT) pres[w] = 0u;
    if (gt < SK_HEAVY) {
      h.heavy_id[gt] = SK_EMPTY;
      h.heavy_n[gt] = 0u;
    }
    for (int w = gt; w < 64; w += GT) h.aux[w] = 0u;
    if (gt == 0) {
      h.status = 0u;
      h.nlist = 0u;
      h.nq = 0u;
      h.ovf = 0u;
      h.token = -1;
    }
  };
  clear_tables();
  __syncthreads();

  for (int64_t row = (int64_t)blockIdx.x * geo.R + grp; row < a.num_rows; row += (int64_t)gridDim.x * geo.R) {
    r.row = row;
    r.p1 = (const uint8_t*)a.logits + (size_t)row * row_bytes;
    r.p2 = CFG ? r.p1 + (size_t)dv.second * row_bytes : r.p1;
    r.idsr = (const uint8_t*)a.input_ids + (size_t)row * (size_t)a.ids_row_stride * ids_esz;
    // the row's logits and history window go to L2 in three bulk prefetches, so
    // the history rounds and the chunk loads below find them there
    const bool need_hist = r.pen_on || (scan_mode && L > 0);
    if (gt == 0) {
      // rows start 16-byte aligned and V % 8 == 0: whole 16-byte granules
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r.p1), "r"((uint32_t)(V * sizeof(Tin))) : "memory");
      if (CFG)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(r.p2), "r"((uint32_t)(V * sizeof(Tin))) : "memory");
      if (need_hist) {
        const int h0 = scan_mode ? 0 : a.penalty_start;
        l2_prefetch(r.idsr + (size_t)h0 * ids_esz, (size_t)(L - h0) * ids_esz);
      }
    }
    constexpr int NBUF = J <= 4 ? J : 2;  // J <= 4: every chunk of the row in flight at once
    uint4 bufA[NBUF][NV], bufB[NBUF][NV];
    if (J > 4 && gt < nch) r.ld_chunk(gt, bufA[0], bufB[0]);

    // ---------------- per-row scalars (every thread, the same addresses)
    uint32_t st = 0;
    int32_t mono = -1;
    if (a.mono_mode == MTR_MONO_STATE) {
      mono = a.mono_state ? a.mono_state[row] : -1;
      if ((a.flags & MTR_FLAG_MONO_UPDATE_FROM_IDS) && L > 0) mono = mono_update(a, mono, r.raw_id(a, L - 1));
    }
    r.gb = nullptr;
    if (a.grammar_class_of) {
      int64_t prev = -1;
      if (a.flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) prev = L > 0 ? r.raw_id(a, L - 1) : -1;
      else if (a.prev_token) prev = a.prev_token[row];
      if (prev >= V) st |= MTR_ROW_BAD_ID;
      if (prev >= 0 && prev < V) {
        const uint32_t c = __ldg(a.grammar_class_of + prev);
        if (c < (uint32_t)a.grammar_n_classes) r.gb = a.grammar_vocab_bits + (size_t)c * dv.gwords;
        else st |= MTR_ROW_BAD_ID;
      }
    }
    r.t_row = a.temperature;
    r.t_rcp = dv.temp_rcp;
    if (a.temp_mode == MTR_TEMP_ROW_CONDITIONAL) {
#pragma unroll 1
      for (int c = 0; c < a.n_cond; ++c) {
        const int off = a.cond_offset[c];
        if (off < 1 || L < off) continue;
        const int64_t tok = r.raw_id(a, L - off);
        if (tok >= 0 && tok < V && ((__ldg(a.cond_token_bits[c] + (tok >> 5)) >> (tok & 31)) & 1u)) {
          r.t_row = a.cond_temperature[c];
          r.t_rcp = dv.cond_rcp[c];
          break;
        }
      }
    }
    r.u = 0.0f;
    if (sample) {
      float u = a.uniforms[row];
      if (!(u >= 0.0f)) {
        u = 0.0f;
        st |= MTR_ROW_BAD_UNIFORM;
      } else if (u >= 1.0f) {
        u = 0x1.fffffep-1f;
        st |= MTR_ROW_BAD_UNIFORM;
      }
      r.u = u;
    }

    // ---------------- history: counts + presence (and the monotonic full scan)
    if (need_hist) {
      const int ps = a.penalty_start;
      bool ovf = false;
      if (scan_mode) {
        // monotonic full scan: the last time shift and the last start-of-sequence
        int last_ts = -1, last_sos = -1;
#pragma unroll 1
        for (int rb = 0; rb < L; rb += GT * SK_HPT) {
          int64_t ids[SK_HPT];
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const int pos = rb + gt + k * GT;
            ids[k] = pos < L ? r.raw_id(a, pos) : -1;
          }
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const int pos = rb + gt + k * GT;
            if (pos >= L) continue;
            if (ids[k] >= a.ts_start && ids[k] < a.ts_end) last_ts = pos;
            if (is_sos(a, ids[k])) last_sos = pos;
          }
        }
        last_ts = g.max_i32(last_ts);
        last_sos = g.max_i32(last_sos);
        mono = (last_ts != -1 && last_ts > last_sos) ? (int32_t)(r.raw_id(a, last_ts) - a.ts_start) : -1;
      }
      if (r.pen_on) {
        // penalty window: counts and presence bits (shared atomics)
#pragma unroll 1
        for (int rb = ps; rb < L; rb += GT * SK_HPT) {
          uint32_t tw[SK_HPT];
          bool ok[SK_HPT];
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const int pos = rb + gt + k * GT;
            ok[k] = false;
            tw[k] = pos < L ? r.id_at(a, pos, ok[k]) : 0u;
          }
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const uint32_t t = tw[k];
            if (ok[k]) {
              if (geo.cnt16) {
                atomicAdd(cnt + (t >> 1), 1u << (16 * (t & 1)));
              } else {
                const uint32_t sh = 8u * (t & 3u);
                const uint32_t old = atomicAdd(cnt + (t >> 2), 1u << sh);
                ovf |= ((old >> sh) & 0xffu) == 0xffu;
              }
              atomicOr(pres + (t >> 5), 1u << (t & 31));
            } else if (rb + gt + k * GT < L) {
              st |= MTR_ROW_BAD_ID;
            }
          }
        }
      }
      if (r.pen_on && !geo.cnt16) {
        // an 8-bit count wrapped (an id repeated 256 times or more): count the
        // window again with saturating updates; counts past 255 go to the
        // heavy table
        if (ovf) h.ovf = 1u;
        g.sync();
        if (h.ovf) {
          g.sync();
          for (int w = gt; w < cnt_words; w += GT) cnt[w] = 0u;
          g.sync();
#pragma unroll 1
          for (int pos = ps + gt; pos < L; pos += GT) {
            const int64_t t = r.raw_id(a, pos);
            if (t < 0 || t >= V) continue;
            const int ti = (int)t;
            uint32_t* w = cnt + (ti >> 2);
            const uint32_t sh = 8u * (uint32_t)(ti & 3);
            uint32_t old = *(volatile uint32_t*)w;
#pragma unroll 1
            for (int tries = 0; tries < (1 << 20); ++tries) {  // each failed CAS is another thread's success
              if (((old >> sh) & 0xffu) == 0xffu) {
#pragma unroll 1
                for (int i = 0; i < SK_HEAVY; ++i) {
                  const uint32_t was = atomicCAS(&h.heavy_id[i], SK_EMPTY, (uint32_t)ti);
                  if (was == SK_EMPTY || was == (uint32_t)ti) {
                    atomicAdd(&h.heavy_n[i], 1u);
                    break;
                  }
                }
                break;
              }
              const uint32_t was = atomicCAS(w, old, old + (1u << sh));
              if (was == old) break;
              old = was;
            }
          }
        }
      }
    }
    g.sync();  // counts and presence complete

    // ---------------- pass 1: chunk maxima of the masked, CFG-combined scores
    r.mono_lo = a.ts_start;
    r.mono_hi = mono >= 0 ? min(a.ts_end, a.ts_start + mono) : a.ts_start;
    // Per chunk an upper bound ub of its largest score (history ids excluded):
    // exact for fp32 logits, 16-bit logits without CFG, or with a timeshift
    // bias; otherwise from the packed approximation, with the row's largest
    // bound half-width W so that ub - 2W is a lower bound of the chunk maximum.
    // A NaN, infinite or huge bound marks the chunk special: it is always read
    // again exactly (which finds the non-finite scores) and never binned.
    const bool approx = sizeof(Tin) == 2 && !r.bias_on && (!CFG || geo.bound_cfg);
    float ub[J];
    float wmax = 0.0f, rmax = NEG;
    if constexpr (J <= 4) {
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (j * GT + gt < nch) r.ld_chunk(j * GT + gt, bufA[j], bufB[j]);
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = j * GT + gt;
      const int s = J <= 4 ? j : (j & 1);
      if (J > 4 && j + 1 < J && c + GT < nch) r.ld_chunk(c + GT, bufA[s ^ 1], bufB[s ^ 1]);
      float m = NEG;
      const uint32_t keep = c < nch ? r.keep_of(c, true) : 0u;
      if (__any_sync(FULL, keep != 0u)) {
        if (approx) {
          float am, um;
          r.chunk_bound(bufA[s], bufB[s], keep, geo.s16x2, geo.m16x2, am, um);
          if (CFG) {
            const bool fin = fabsf(am) < 0x1p126f && um < 0x1p126f;  // false for NaN
            const float w = __fmaf_ru(geo.kappa, fabsf(am), __fmaf_ru(geo.lambda, um, geo.bound_abs));
            m = fin ? __fadd_ru(am, w) : (keep ? pos_inf() : NEG);
            if (fin && keep) wmax = fmaxf(wmax, w);
          } else {
            m = am != am ? pos_inf() : am;  // exact; NaN: special
          }
          if (!keep) m = NEG;
        } else {
          float y[8];
          r.chunk_y(bufA[s], bufB[s], keep, y);
          if (r.bias_on) r.add_bias(a, y, 8 * c);
          m = sk_max8(y);
        }
      }
      ub[j] = m;
      if (!approx || m < pos_inf()) rmax = fmax2n(rmax, m);
    }
    // exact path: any NaN or +inf makes the row non-finite; the bounded path
    // finds non-finite scores when it reads the special chunks again
    const bool rnan = rmax != rmax;
    const bool any_nan = g.or_u32(rnan ? 1u : 0u) != 0u;
    const float Ms = key2f(g.max_u32(rnan ? 0u : fkey(rmax)));
    const float W2 = approx && CFG ? __fmul_ru(2.0f, __uint_as_float(g.max_u32(__float_as_uint(wmax)))) : 0.0f;
    bool clean = approx ? true : !(any_nan || Ms == pos_inf());
    if (!clean) st |= MTR_ROW_NONFINITE;

    // ---------------- bound: k chunk maxima above T
    float lower = NEG;
    if (clean && Ms > NEG) {
      float scale = 8.0f;
#pragma unroll 1
      for (int lvl = 0; lvl < 2; ++lvl) {
#pragma unroll
        for (int j = 0; j < J; ++j) {
          if (ub[j] > NEG && ub[j] < pos_inf()) {
            // bin of the chunk's lower bound lb = RD(ub - W2) (<= its largest score):
            // bin <= b* implies Ms - lb < (b* + 1) / scale, i.e. lb > T
            const float lb = __fsub_rd(ub[j], W2);
            const float d = __fmul_rn(__fsub_rn(Ms, lb), scale);
            atomicAdd(&h.aux[__float2int_rz(fminf(d, 63.0f))], 1u);
          }
        }
        g.sync();
        if (g.wig == 0) {
          const uint32_t c0 = h.aux[2 * lane], c1 = h.aux[2 * lane + 1];
          const uint32_t incl = warp_incl_scan_u32(c0 + c1, lane);
          const uint32_t excl = incl - c0 - c1;
          const uint32_t k = (uint32_t)r.k_top;
          int b = -1;
          if (excl < k && excl + c0 >= k) b = 2 * lane;
          else if (excl + c0 < k && incl >= k) b = 2 * lane + 1;
          const unsigned bal = __ballot_sync(FULL, b >= 0);
          int bs = bal ? __shfl_sync(FULL, b, __ffs(bal) - 1) : -1;
          if (bs >= 63) bs = -1;  // the overflow bin bounds nothing
          __syncwarp();
          h.aux[2 * lane] = 0u;
          h.aux[2 * lane + 1] = 0u;
          if (lane == 0) h.bstar = bs;
        }
        g.sync();
        const int bstar = h.bstar;
        g.sync();
        if (bstar >= 0) {
          lower = __fsub_rd(Ms, (float)(bstar + 1) / scale);
          break;
        }
        scale = 1.0f;
      }
      if (r.t_row != 1.0f && lower > NEG)
        lower = __fsub_rd(__fsub_rd(lower, __fmul_ru(fabsf(lower), 0x1p-20f)), geo.margin_abs);
    }

    if (clean) {
      // ---------------- listing: chunks whose maximum reaches the bound
      uint32_t qm = 0;
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (ub[j] > NEG && ub[j] >= lower) qm |= 1u << j;  // special chunks (+inf) always
      const uint32_t nqt = __popc(qm);
      const uint32_t qincl = warp_incl_scan_u32(nqt, lane);
      const uint32_t qtot = __shfl_sync(FULL, qincl, 31);
      uint32_t qbase = 0;
      if (g.G > 1) {
        if (lane == 31) qbase = atomicAdd(&h.nq, qtot);
        qbase = __shfl_sync(FULL, qbase, 31);
      }
      uint16_t* qc = (uint16_t*)h.aux;
      {
        uint32_t slot = qbase + qincl - nqt, m = qm;
        while (m) {
          const int j = __ffs(m) - 1;
          m &= m - 1u;
          if (slot < (uint32_t)SK_QCAP) qc[slot] = (uint16_t)(j * GT + gt);
          ++slot;
        }
      }
      g.sync();
      const uint32_t nq = g.G > 1 ? h.nq : qtot;
      auto list_chunk = [&](int c, bool act) __attribute__((always_inline)) {
        float y[8];
        uint32_t sel = 0;
        if (act) {
          uint4 ra[NV], rb[NV];
          r.ld_chunk_l2(c, ra, rb);
          r.chunk_y(ra, rb, r.keep_of(c, true), y);
          if (r.bias_on) r.add_bias(a, y, 8 * c);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (y[e] > NEG && y[e] >= lower) sel |= 1u << e;
          const float ym = sk_max8(y);
          if (ym != ym || ym == pos_inf()) st |= MTR_ROW_NONFINITE;
          if (sel && r.t_row != 1.0f) {
            div_chunk(y, r.t_row, r.t_rcp);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (((sel >> e) & 1u) && y[e] == pos_inf()) st |= MTR_ROW_NONFINITE;
          }
        }
        r.append(sel, y, 8 * c);
      };
      if (nq <= (uint32_t)SK_QCAP) {
#pragma unroll 1
        for (uint32_t b0 = 0; b0 < nq; b0 += (uint32_t)GT) {
          const uint32_t i = b0 + (uint32_t)gt;
          const bool act = i < nq;
          list_chunk(act ? (int)qc[i] : 0, act);
        }
      } else {
#pragma unroll 1
        for (int j = 0; j < J; ++j) list_chunk(j * GT + gt, ((qm >> j) & 1u) != 0u);
      }

      // ---------------- history ids: penalised scores
      if (r.pen_on) {
        const float rp = a.repetition_penalty, fp = a.frequency_penalty, pp = a.presence_penalty;
#pragma unroll 1
        for (int rb = a.penalty_start; rb < L; rb += GT * SK_HPT) {
          uint32_t tw[SK_HPT];
          bool ok[SK_HPT];
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const int pos = rb + gt + k * GT;
            ok[k] = false;
            tw[k] = pos < L ? r.id_at(a, pos, ok[k]) : 0u;
          }
          // scores of the window ids before penalties, branch-free (invalid ids read id 0)
          float c1[SK_HPT], c2[SK_HPT];
          uint32_t gw[SK_HPT];
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const uint32_t tt = ok[k] ? tw[k] : 0u;
            gw[k] = r.gb ? __ldg(r.gb + (tt >> 5)) : 0xffffffffu;
            c1[k] = T::one(r.p1, (int)tt);
            c2[k] = CFG ? T::one(r.p2, (int)tt) : 0.0f;
          }
          uint32_t cand = 0;
          float yr[SK_HPT];
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            const uint32_t tt = ok[k] ? tw[k] : 0u;
            float y = c1[k];
            if (CFG) y = __fmaf_rn(__fmaf_rn(__fmaf_rn(c2[k], dv.neg_one, c1[k]), a.cfg_scale, dv.neg_zero), dv.one, c2[k]);
            if (r.bias_on && tt >= (uint32_t)a.ts_start && tt < (uint32_t)a.ts_end) y = __fadd_rn(y, a.timeshift_bias);
            const bool kept = ok[k] && ((gw[k] >> (tt & 31)) & 1u) &&
                              (tt - (uint32_t)r.mono_lo) >= (uint32_t)(r.mono_hi - r.mono_lo);
            yr[k] = kept ? y : NEG;
            if (ok[k] && (!(yr[k] < lower) || !geo.pen_fast)) cand |= 1u << k;
          }
          // candidates: claim the id (first of its occurrences), penalties, temperature
          float xs[SK_HPT];
          int ts[SK_HPT];
          uint32_t sel = 0;
#pragma unroll
          for (int k = 0; k < SK_HPT; ++k) {
            xs[k] = NEG;
            ts[k] = (int)tw[k];
            if ((cand >> k) & 1u) {
              const uint32_t ti = tw[k];
              const uint32_t bit = 1u << (ti & 31);
              const uint32_t was = atomicAnd(pres + (ti >> 5), ~bit);
              if (was & bit) {
                float yp = pen_value(yr[k], (float)r.count_of((int)ti), rp, fp, pp, dv.rep_rcp);
                if (yp != yp || yp == pos_inf()) {
                  st |= MTR_ROW_NONFINITE;
                } else if (yp > NEG && yp >= lower) {
                  if (r.t_row != 1.0f) yp = div_by(yp, r.t_row, r.t_rcp);
                  if (yp == pos_inf()) st |= MTR_ROW_NONFINITE;
                  xs[k] = yp;
                  sel |= 1u << k;
                }
              }
            }
          }
          r.append(sel, xs, 0, ts);
        }
      }
    }

    // ---------------- status so far; the row is clean, all masked, or to be selected
    st = g.or_u32(st);
    clean = !(st & MTR_ROW_NONFINITE);
    g.sync();
    const uint32_t nl = h.nlist;
    if (clean && nl == 0u) st |= MTR_ROW_ALL_MASKED;
    const bool select_row = clean && nl > 0u;
    SkSel s;
    s.mode = 0;
    s.kcut = 0;
    s.qkept = 0;
    s.target = 0;
    s.mx = NEG;
    s.kth = 0;
    s.nstar = 0;
    s.token = -1;
    const bool slow = select_row && (nl > (uint32_t)SK_CAP || (a.flags & MTR_FLAG_FORCE_RADIX));
    if (select_row && !slow) {
      if (g.wig == 0) sk_select_list(r, a, geo.bucket_shift, (int)nl, sample, topp_on);
      g.sync();
      s.token = h.token;
      s.kcut = h.bc[0];
      s.mx = __uint_as_float((uint32_t)h.bc[1]);
      s.qkept = h.bc[2];
    } else if (slow) {
      st |= MTR_ROW_SLOW_PATH;
      SkRow<Tin, CFG> rc = r;
      sk_slow_select(rc, a, dv, geo.bucket_shift, sample, topp_on, &s);
    }

    // ---------------- walk in id order: outputs, and the draw of the tie mode
    const bool draw_walk = s.mode == 1 && sample;
    if (want_out || draw_walk) {
      SkRow<Tin, CFG> rc = r;
      if (draw_walk && gt == 0) h.token = -1;
      g.sync();
      sk_walk(rc, a, dv, s, select_row, draw_walk);
      if (draw_walk) s.token = h.token;
    }

    // ---------------- epilogue
    st = g.or_u32(st);
    if (gt == 0) {
      uint32_t status = st | h.status;
      if (a.select_mode != MTR_SELECT_NONE) {
        const int64_t tok =
            finish_token(a, row, (select_row && s.token >= 0) ? (int64_t)s.token : a.pad_id, &status);
        if (a.flags & MTR_FLAG_MONO_UPDATE_FROM_SAMPLE) mono = mono_update(a, mono, tok);
        if ((a.flags & MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE) && a.prev_token) a.prev_token[row] = (int32_t)tok;
        if (a.out_ids) a.out_ids[row] = tok;
      }
      if (a.mono_mode != MTR_MONO_OFF && a.mono_state) a.mono_state[row] = mono;
      if (a.out_status) a.out_status[row] = status;
    }
    g.sync();
    clear_tables();
    g.sync();
  }
}

// Per element type (mtr_stream_{bf16,f16,f32}.cu): the kernel of (cfg, shape)
// and its launch.
const void* stream_kernel_bf16(bool cfg, int shape, bool j4);
const void* stream_kernel_f16(bool cfg, int shape, bool j4);
const void* stream_kernel_f32(bool cfg, int shape, bool j4);
cudaError_t stream_launch_bf16(const MtrSamplerArgs& a, const Derived& d, const SkGeo& g, const SkLaunch& sh,
                               cudaStream_t s);
cudaError_t stream_launch_f16(const MtrSamplerArgs& a, const Derived& d, const SkGeo& g, const SkLaunch& sh,
                              cudaStream_t s);
cudaError_t stream_launch_f32(const MtrSamplerArgs& a, const Derived& d, const SkGeo& g, const SkLaunch& sh,
                              cudaStream_t s);

// The instantiations of one element type: shapes 128 (7 CTAs / SM), 256 (3) and
// 512 (2 CTAs / SM) threads.
#define MTR_STREAM_KERNEL(TIN, C, SHAPE, J4)                                                                    \
  ((SHAPE) == SK_SHAPE_128 ? ((J4) ? (const void*)stream_kernel<TIN, C, 128, 7, 4>                              \
                                   : (const void*)stream_kernel<TIN, C, 128, 7, SK_J>)                          \
   : (SHAPE) == SK_SHAPE_256 ? ((J4) ? (const void*)stream_kernel<TIN, C, 256, 3, 4>                            \
                                     : (const void*)stream_kernel<TIN, C, 256, 3, SK_J>)                        \
   : ((J4) ? (const void*)stream_kernel<TIN, C, 512, 2, 4> : (const void*)stream_kernel<TIN, C, 512, 2, SK_J>))

#define MTR_STREAM_INSTANTIATE(TIN, NAME)                                                                        \
  const void* stream_kernel_##NAME(bool cfg, int shape, bool j4) {                                              \
    return cfg ? MTR_STREAM_KERNEL(TIN, true, shape, j4) : MTR_STREAM_KERNEL(TIN, false, shape, j4);            \
  }                                                                                                               \
  cudaError_t stream_launch_##NAME(const MtrSamplerArgs& a, const Derived& d, const SkGeo& g, const SkLaunch& sh, \
                                   cudaStream_t s) {                                                             \
    cudaLaunchConfig_t cfg;                                                                                       \
    memset(&cfg, 0, sizeof(cfg));                                                                                 \
    cfg.gridDim = dim3((unsigned)sh.grid, 1, 1);                                                                  \
    cfg.blockDim = dim3((unsigned)sh.threads, 1, 1);                                                              \
    cfg.dynamicSmemBytes = (size_t)sh.dyn;                                                                        \
    cfg.stream = s;                                                                                               \
    cudaLaunchAttribute attr[2];                                                                                  \
    cfg.numAttrs = launch_attrs(attr, 1, d.pdl != 0);                                                             \
    cfg.attrs = cfg.numAttrs ? attr : nullptr;                                                                    \
    const void* kern = stream_kernel_##NAME(a.cfg_enabled != 0, sh.shape, sh.j4 != 0);                           \
    void* params[3] = {(void*)&a, (void*)&d, (void*)&g};                                                         \
    return cudaLaunchKernelExC(&cfg, kern, params);                                                               \
  }

}  // namespace mtr
