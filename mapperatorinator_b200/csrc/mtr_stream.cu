// mtr_stream.cu -- host side of the streaming row-group kernel (mtr_stream.cuh):
// which requests it serves, its row-group geometry, launch and query.
#include "mtr_stream.cuh"

namespace mtr {

bool sk_supported(const MtrSamplerArgs& a, const Derived& d) {
  if (a.select_mode == MTR_SELECT_ARGMAX) return false;
  if (a.lookback_mode != MTR_LOOKBACK_OFF) return false;
  if (a.top_k < 1 || a.top_k > SK_TOPK_MAX || a.top_k >= a.vocab) return false;
  if (a.vocab % 8 != 0 || a.vocab > SK_MAX_VOCAB) return false;
  if (!d.vec_ok) return false;
  if (a.temp_mode == MTR_TEMP_COLUMN_RANGES) return false;
  if (a.grammar_class_of && !a.grammar_vocab_bits) return false;
  return true;
}

static int align16(int v) { return (v + 15) & ~15; }

static uint16_t bf16_rn_bits(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static double bf16_bits_value(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

// Constants of the packed CFG bound (16-bit logits).  With s16 = RN16(s),
// m16 = RN16(1 - s), rho the unit roundoff of the 16-bit type and fp32's 2^-24,
// the packed a = RN16(c s16 + RN16(u m16)) of an element (c, u) and its exact
// fp32 CFG value f = RN(u + RN(RN(c - u) s)) satisfy
//   |a - f| <= kappa |a| + lambda |u| + abs,
// where |c| is bounded through a and u (c s16 = a / (1 + e) - t):
//   kappa  = (1+2^-20) (rho (1+2rho) + (1+2rho)(ds + 2^-23 s) / s16 + 2^-23)
//   lambda = (1+2^-20) ((1+rho)|m16|(ds + 2^-23 s) / s16 + rho |m16| + dm + 2^-23 s)
// (ds = |s - s16|, dm = |1 - s - m16|; abs covers flushed subnormals).  Both
// are rounded up by 1%.  Scales whose 16-bit rounding is not positive and
// finite keep the exact chunk maxima.
static void sk_bound_constants(const MtrSamplerArgs& a, SkGeo* g) {
  g->bound_cfg = 0;
  g->kappa = g->lambda = g->bound_abs = 0.0f;
  g->s16x2 = g->m16x2 = 0u;
  if (!a.cfg_enabled || (a.logits_dtype != MTR_DTYPE_BF16 && a.logits_dtype != MTR_DTYPE_F16)) return;
  const double s = (double)a.cfg_scale, m = 1.0 - s;
  uint16_t sb, mb;
  double s16, m16, rho, absr;
  if (a.logits_dtype == MTR_DTYPE_BF16) {
    sb = bf16_rn_bits((float)s);
    mb = bf16_rn_bits((float)m);
    s16 = bf16_bits_value(sb);
    m16 = bf16_bits_value(mb);
    rho = 0x1p-8;
    absr = 0x1p-118;
  } else {
    const __half hs = __float2half_rn((float)s), hm = __float2half_rn((float)m);
    sb = __half_as_ushort(hs);
    mb = __half_as_ushort(hm);
    s16 = (double)__half2float(hs);
    m16 = (double)__half2float(hm);
    rho = 0x1p-11;
    absr = 0x1p-20;
  }
  if (!(s16 > 0.0 && s16 < 1e30 && fabs(m16) < 1e30)) return;
  const double e23 = 0x1p-23, ds = fabs(s - s16), dm = fabs(m - m16);
  const double kappa = (1.0 + 0x1p-20) * (rho * (1 + 2 * rho) + (1 + 2 * rho) * (ds + e23 * s) / s16 + e23);
  const double lambda =
      (1.0 + 0x1p-20) * ((1 + rho) * fabs(m16) * (ds + e23 * s) / s16 + rho * fabs(m16) + dm + e23 * s);
  g->bound_cfg = 1;
  g->s16x2 = (uint32_t)sb | ((uint32_t)sb << 16);
  g->m16x2 = (uint32_t)mb | ((uint32_t)mb << 16);
  g->kappa = (float)(kappa * 1.01);
  g->lambda = (float)(lambda * 1.01);
  g->bound_abs = (float)(absr * (s16 > 1.0 ? s16 : 1.0) * 4.0);
}

// Row-group geometry: the fewest warps per row that cover the vocabulary with
// SK_J chunks per thread, doubled while the rows would leave more than half of
// the device's warp slots empty (few rows: more warps per row, shorter rows).
static SkGeo sk_geo(const MtrSamplerArgs& a, const Derived& d, int sms) {
  SkGeo g;
  memset(&g, 0, sizeof(g));
  const int V = a.vocab;
  int G = 1;
  while (256 * SK_J * G < V) G *= 2;
  const int64_t slots = (int64_t)sms * 28;  // resident warps of the 128-thread shape
  while (G < SK_MAX_G && (int64_t)a.num_rows * G * 2 <= slots) G *= 2;
  g.G = G;
  g.R = G >= 4 ? 1 : 4 / G;
  const int lpen = d.pen_on ? a.ids_len - a.penalty_start : 0;
  g.cnt16 = lpen >= 256 * SK_HEAVY;
  g.cnt_off = (int)sizeof(SkHead);
  g.pres_off = g.cnt_off + align16(V * (g.cnt16 ? 2 : 1));
  g.group_bytes = g.pres_off + align16((V + 31) / 32 * 4);
  g.pen_fast = a.repetition_penalty >= 1.0f && a.frequency_penalty >= 0.0f && a.presence_penalty >= 0.0f;
  int bits = 0;
  while ((1 << bits) < V) ++bits;
  g.bucket_shift = bits > 5 ? bits - 5 : 0;
  g.margin_abs = 0x1p-100f;
  sk_bound_constants(a, &g);
  return g;
}

static const void* stream_kernel_for(const MtrSamplerArgs& a, int shape, bool j4) {
  const bool cfg = a.cfg_enabled != 0;
  switch (a.logits_dtype) {
    case MTR_DTYPE_F32: return stream_kernel_f32(cfg, shape, j4);
    case MTR_DTYPE_BF16: return stream_kernel_bf16(cfg, shape, j4);
    default: return stream_kernel_f16(cfg, shape, j4);
  }
}

// Launch shape of the stream kernel: threads per CTA pick the instantiation
// (128: 7 CTAs per SM, 256: 3, 512: 2); the kernel attribute for large dynamic
// shared memory is set once per device and instantiation.
static cudaError_t sk_shape(const MtrSamplerArgs& a, const SkGeo& g, int sms, SkLaunch* out) {
  out->threads = g.R * g.G * 32;
  out->shape = out->threads <= 128 ? SK_SHAPE_128 : out->threads <= 256 ? SK_SHAPE_256 : SK_SHAPE_512;
  out->dyn = SK_LUT_BYTES + g.R * g.group_bytes;
  out->j4 = (int64_t)4 * 256 * g.G >= (int64_t)a.vocab;
  const void* kern = stream_kernel_for(a, out->shape, out->j4 != 0);
  {
    static std::mutex mu;
    static const void* done[64][36];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(mu);
    bool set = false;
    for (int i = 0; i < 36; ++i) set |= done[dev][i] == kern;
    if (!set) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (e != cudaSuccess) return e;
      for (int i = 0; i < 36; ++i)
        if (!done[dev][i]) {
          done[dev][i] = kern;
          break;
        }
    }
  }
  int occ = 0;
  const cudaError_t e = cached_occupancy(kern, out->threads, out->dyn, &occ);
  if (e != cudaSuccess) return e;
  const int64_t ctas = ((int64_t)a.num_rows + g.R - 1) / g.R;
  const int64_t cap = (int64_t)occ * sms;
  out->grid = (int)(ctas < cap ? ctas : cap);
  return cudaSuccess;
}

cudaError_t stream_launch(const MtrSamplerArgs& a, const Derived& d, int sms, cudaStream_t s) {
  const SkGeo g = sk_geo(a, d, sms);
  SkLaunch sh{};
  const cudaError_t e = sk_shape(a, g, sms, &sh);
  if (e != cudaSuccess) return e;
  switch (a.logits_dtype) {
    case MTR_DTYPE_F32: return stream_launch_f32(a, d, g, sh, s);
    case MTR_DTYPE_BF16: return stream_launch_bf16(a, d, g, sh, s);
    default: return stream_launch_f16(a, d, g, sh, s);
  }
}

void stream_query(const MtrSamplerArgs& a, const Derived& d, int sms, MtrLaunchInfo* out) {
  const SkGeo g = sk_geo(a, d, sms);
  SkLaunch sh{};
  if (sk_shape(a, g, sms, &sh) != cudaSuccess) {
    cudaGetLastError();  // no device: report the launch bound (28 warps per SM)
    sh.threads = g.R * g.G * 32;
    sh.dyn = SK_LUT_BYTES + g.R * g.group_bytes;
    const int64_t ctas = ((int64_t)a.num_rows + g.R - 1) / g.R;
    const int64_t cap = (int64_t)(sh.threads <= 128 ? 7 : sh.threads <= 256 ? 3 : 2) * sms;
    sh.grid = (int)(ctas < cap ? ctas : cap);
  }
  out->threads = sh.threads;
  out->elems_per_thread = 8 * (sh.j4 ? 4 : SK_J);
  out->cluster_size = 1;
  out->grid = sh.grid;
  out->dyn_smem_bytes = sh.dyn;
  out->max_vocab = MTR_MAX_VOCAB;
  out->max_ids_len = MTR_MAX_IDS_LEN;
  out->candidate_cap = SK_CAP;
  out->kernel = 2;
}

}  // namespace mtr
