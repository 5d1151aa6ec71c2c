// mtr_sampler.cu -- fused decode-sampling step for sm_100a (B200).
//
// One output row of the [B, V] processed logits is owned by one CTA, or by a
// thread-block cluster of CS CTAs (large V, or few rows).  The row lives in
// registers (THREADS x EPT elements per CTA) from the first 128-bit load to the
// last store; no intermediate B x V tensor ever reaches HBM.  The step is
// instruction-bound long before it is HBM-bound, so every per-element
// operation is counted: feature switches are hoisted out of the element loops,
// arithmetic on element pairs uses the packed f32x2 instructions of sm_100a
// (bit-identical per lane to the scalar IEEE operations), masks are built once
// per 8-element chunk, and the selection stages work on short lists.
//
//   prologue   monotonic state (stateful, or a full scan of input_ids), grammar
//              row of the previous token, per-row temperature and uniform --
//              independent load chains on separate lanes of warp 0
//   load       ld.global.cs 16-byte vectors of bf16 / f16 / f32 logits; with
//              CFG the first-half row and its second-half partner
//   chain      CFG -> monotonic mask -> timeshift bias -> grammar mask ->
//              penalties (history side, shared-memory histogram) ->
//              temperature (Markstein division, bit-exact to IEEE x / T)
//   stats      max, NaN / +inf detection (arg-max only for greedy selection)
//   top-k      a 1024-bin histogram of the per-thread maxima over d = max - x
//              bounds the k-th value from below (>= k elements lie above it);
//              the elements above that bound are compacted to a list and a
//              second histogram over the list resolves the exact k-th value.
//              Fallback: a histogram over every element
//   top-p      fixed-point probabilities q = floor(e^(x - max) * 2^31), integer
//              sums (keep set independent of thread order); a mass histogram
//              over the survivor list (or over every element when the
//              survivors are many) and an exact resolution inside the crossing
//              bin; ties at the cut go to the lowest token id
//   draw       smallest id whose kept-mass prefix exceeds floor(u * Q_kept):
//              an id-binned mass histogram over the kept list, or per-chunk
//              sums and a block scan over every element
//   epilogue   ids, processed scores / log-probs, row status, state updates
//
// Reference arithmetic followed (paths inside the Mapperatorinator project,
// "HF:" = transformers/generation/):
//   CFG        HF:logits_process.py:2160-2174 (first half = "cond")
//   monotonic  osuT5/osuT5/inference/logit_processors.py:190-229,
//              osuT5/osuT5/inference/optimized/single/logits.py:33-105
//   bias       logit_processors.py:35-43
//   penalty    HF:logits_process.py:407-413 (repetition)
//   temp       HF:logits_process.py:297-301, logit_processors.py:75-119
//   top-k/p    HF:logits_process.py:521-535, 581-588;
//              osuT5/osuT5/inference/compiled_decode.py:1135-1158
//   draw       osuT5/osuT5/inference/optimized/single/decode_loop.py:296-305
//
// The kernel holds no spin-waits: every barrier is __syncthreads() or a
// hardware cluster barrier that all CTAs of the cluster reach on the same,
// row-uniform control path.
#include "mtr_common.cuh"

#include <mutex>

namespace cg = cooperative_groups;

namespace mtr {

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

struct Cross {
  int32_t bin;   // first bin whose inclusive prefix exceeds the limit (-1: none)
  int32_t pad;
  u64 above;     // weight of the bins before it
  u64 w;         // weight of that bin
  u64 total;     // weight of all bins
};

// Warp 0 scans NBINS weights (bin 0 ranks first) and finds the first bin whose
// inclusive prefix exceeds `lim`.  Every thread must call; the result is
// published in *out after the barrier.
template <int NBINS, typename W>
__device__ __forceinline__ void find_crossing(const W* w, u64 lim, Cross* out) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < 32) {
    constexpr int PER = NBINS / 32;
    u64 s = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) s += (u64)w[lane * PER + ((i + lane) & (PER - 1))];  // rotated: no bank conflicts
    const u64 incl = warp_incl_scan_u64(s, lane);
    const u64 excl = incl - s;
    const u64 total = __shfl_sync(FULL, incl, 31);
    if (lane == 0) {
      out->bin = -1;
      out->above = total;
      out->w = 0;
      out->total = total;
    }
    __syncwarp();
    // the crossing lane's segment, resolved by the whole warp (PER <= 32 bins)
    const unsigned bal = __ballot_sync(FULL, excl <= lim && lim < incl);
    if (bal) {
      const int src = __ffs(bal) - 1;
      const u64 seg_excl = __shfl_sync(FULL, excl, src);
      const u64 wi = lane < PER ? (u64)w[src * PER + lane] : 0ull;
      const u64 in2 = warp_incl_scan_u64(wi, lane) + seg_excl;
      const unsigned b2 = __ballot_sync(FULL, lane < PER && in2 > lim);
      const int l2 = __ffs(b2) - 1;  // the first such bin exists: lim < the segment's end
      if (lane == l2) {
        out->bin = src * PER + lane;
        out->above = in2 - wi;
        out->w = wi;
      }
    }
  }
  __syncthreads();
}

// The same for the top-p cut: warp 0 sums the bins, derives the limit from the
// total (P = top_p * total; HF: ceil(P) - 1, sample_fn: floor(P)) and finds its
// crossing in one pass; out->total holds the total, out->pad the mode used.
template <int NBINS, typename WF>
__device__ __forceinline__ void find_topp_crossing(WF w, float top_p, int top_p_mode, Cross* out, u64* plim_out) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < 32) {
    constexpr int PER = NBINS / 32;
    u64 s = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) s += w(lane * PER + ((i + lane) & (PER - 1)));  // rotated: no bank conflicts
    const u64 incl = warp_incl_scan_u64(s, lane);
    const u64 excl = incl - s;
    const u64 total = __shfl_sync(FULL, incl, 31);
    const double P = __dmul_rn((double)top_p, (double)total);
    const u64 lim = top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
    if (lane == 0) {
      out->bin = -1;
      out->above = total;
      out->w = 0;
      out->total = total;
      *plim_out = lim;
    }
    __syncwarp();
    const unsigned bal = __ballot_sync(FULL, excl <= lim && lim < incl);
    if (bal) {
      const int src = __ffs(bal) - 1;
      const u64 seg_excl = __shfl_sync(FULL, excl, src);
      const u64 wi = lane < PER ? w(src * PER + lane) : 0ull;
      const u64 in2 = warp_incl_scan_u64(wi, lane) + seg_excl;
      const unsigned b2 = __ballot_sync(FULL, lane < PER && in2 > lim);
      const int l2 = __ffs(b2) - 1;
      if (lane == l2) {
        out->bin = src * PER + lane;
        out->above = in2 - wi;
        out->w = wi;
      }
    }
  }
  __syncthreads();
}

// The same result with every warp of the CTA: warp w sums bins w*PW ..
// (NBINS/THREADS per lane), the warp totals go through shared memory (`wtot`,
// NW entries), and every warp scans them to find the crossing warp, whose lane
// then resolves its bins.  Two barriers instead of one, but no warp walks more
// than NBINS/THREADS bins.
template <int NBINS, int THREADS, typename WF>
__device__ __forceinline__ void find_topp_crossing_blk(WF w, float top_p, int top_p_mode, Cross* out, u64* plim_out,
                                                       u64* wtot) {
  constexpr int NW = THREADS / 32, BPL = NBINS / THREADS;
  static_assert(NBINS % THREADS == 0 && NW <= 32, "bins per lane");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b0 = tid * BPL;  // this lane's bins, in order
  u64 wb[BPL], s = 0;
#pragma unroll
  for (int i = 0; i < BPL; ++i) {
    wb[i] = w(b0 + i);
    s += wb[i];
  }
  const u64 incl = warp_incl_scan_u64(s, lane);
  if (lane == 31) wtot[warp] = incl;
  __syncthreads();
  const u64 wv = lane < NW ? wtot[lane] : 0ull;
  const u64 winc = warp_incl_scan_u64(wv, lane);
  const u64 total = __shfl_sync(FULL, winc, NW - 1);
  const u64 wbase = __shfl_sync(FULL, winc - wv, warp);
  const double P = __dmul_rn((double)top_p, (double)total);
  const u64 lim = top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
  if (tid == 0) {
    *plim_out = lim;
    out->total = total;
  }
  const u64 lo = wbase + incl - s;
  bool none = !(lim < total);
  if (!none && lo <= lim && lim < lo + s) {  // exactly one lane holds the crossing
    u64 a = lo;
#pragma unroll
    for (int i = 0; i < BPL; ++i) {
      if (a <= lim && lim < a + wb[i]) {
        out->bin = b0 + i;
        out->above = a;
        out->w = wb[i];
      }
      a += wb[i];
    }
  }
  if (tid == 0 && none) {
    out->bin = -1;
    out->above = total;
    out->w = 0;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// shared memory
// ---------------------------------------------------------------------------
struct alignas(16) StatX {  // per-CTA row statistics exchanged across the cluster
  float mx;
  int32_t amax;
  uint32_t nan;
  uint32_t status;
};

template <int CS>
struct alignas(16) Shared {
  // prologue results
  int32_t mono;
  int32_t mono_hi;
  uint32_t allow;
  int32_t grammar_on;
  const uint32_t* gbits;  // vocabulary bitmap of the previous token's class
  float t_row;
  float t_rcp;
  float u;
  uint32_t status;    // bits raised while processing this CTA's tile
  uint32_t status_g;  // grammar lookups
  uint32_t status_u;  // uniform
  uint32_t warm;      // see the parameter warm-up in the prologue
  int32_t n_uniq;
  int32_t nc;         // local candidate count
  int32_t nm;         // crossing-bin list count
  int32_t token;
  int32_t red_i[2];
  float tk;
  uint32_t nsurv;
  float cut_x;
  int32_t cut_id;
  u64 qtot;
  u64 qkept;
  u64 plim;  // top-p limit published by find_topp_crossing
  Cross cr;
  StatX stat;
  u64 cta_mass;
  uint32_t cta_nfin;
  // lookback bias (renormalising form)
  StatX lbx;       // this CTA's maximum and non-finite flag of the scores before the bias
  u64 lbs[3];      // this CTA's masses Q, O, E
  double lb_c;     // scores outside the range become x - lb_c
  float lb_v;      // the score of lb_start
  float lb_new;    // the row's next lb_state
  float lb_p;      // the row's lb_state on entry
  int32_t lb_timed;  // the last input id is a timed-event token
  int32_t lb_do;     // apply the transform
  // per-warp partials
  float wf[32];
  int32_t wi[32];
  int32_t wi2[32];
  uint32_t wu[32];
  uint32_t wu2[32];
  u64 wl[32 * 4];
  // histograms (local; merged copies when CS > 1)
  uint32_t hcnt[NB];
  alignas(16) u64 hmass[NB];
  uint32_t hcnt_m[CS > 1 ? NB : 1];
  u64 hmass_m[CS > 1 ? NB : 1];
  // candidate lists (local; merged when CS > 1)
  float cx[CAP];
  int32_t cid[CAP];
  uint32_t cq[CAP];
  int32_t cb[CAP];
  float mcx[CS > 1 ? CAP : 1];
  int32_t mcid[CS > 1 ? CAP : 1];
  uint32_t mcq[CS > 1 ? CAP : 1];
  // crossing-bin list
  float nx[MINI];
  int32_t nid[MINI];
  uint32_t nq[MINI];
  uint8_t ckeep[CAP];
  uint32_t gword[512];  // this CTA's words of the previous token's grammar bitmap (tile / 32 <= 512)
};


// Push the elements of this thread whose bit is set in `mask` to the local
// candidate list (x, id, q): a warp scan of the counts and one shared atomic per
// warp.  Every lane of the warp must call.  Entries past CAP are counted only.
template <int CS, int EPT, typename IdOf>
__device__ __forceinline__ void collect(Shared<CS>& sm, uint32_t mask, const float (&x)[EPT], const uint32_t (&q)[EPT],
                                        bool with_q, IdOf id_of, int lane) {
  const uint32_t c = __popc(mask);
  const uint32_t incl = warp_incl_scan_u32(c, lane);
  const uint32_t wt = __shfl_sync(FULL, incl, 31);
  if (wt == 0u) return;
  int base = 0;
  if (lane == 31) base = atomicAdd(&sm.nc, (int)wt);
  base = __shfl_sync(FULL, base, 31);
  if (mask) {
    int s = base + (int)(incl - c);
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      if ((mask >> k) & 1u) {
        if (s < CAP) {
          sm.cx[s] = x[k];
          sm.cid[s] = id_of(k);
          sm.cq[s] = with_q ? q[k] : 0u;
        }
        ++s;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Residency (MINB): three CTAs per SM for one 256-thread CTA per row (80
// registers, no spills), four in the instantiation for launches of more rows
// than one round of three holds (64 registers, a few spilled: 1024 top-p-only
// rows run 9 % faster than at three, but rows that fit one round run up to 19 %
// slower, so they keep three), two for the 256-thread clusters (which would
// spill at three), one for the wider CTAs.
template <typename Tin, int THREADS, int EPT, int CS, int MINB = (THREADS <= 256 ? (CS == 1 ? 3 : 2) : 1)>
__global__ void __launch_bounds__(THREADS, MINB)
    sampler_kernel(const __grid_constant__ MtrSamplerArgs a, const __grid_constant__ Derived dv) {
  wait_prior_grid();
  allow_dependents();
  using E = Elem<Tin>;
  constexpr int VEC = E::VEC;
  constexpr int NCH = EPT / VEC;
  constexpr int TILE = THREADS * EPT;
  constexpr int NW = THREADS / 32;
  static_assert(EPT % VEC == 0 && VEC % 2 == 0, "EPT must be a multiple of the (even) vector width");
  static_assert(EPT <= 32, "per-thread element masks are 32 bits");
  static_assert(THREADS >= CAP, "one thread per list entry");
  static_assert(NCH <= 4, "per-chunk partials");
  static_assert(TILE <= (1 << 14), "the split u32 mass histogram holds <= 2^14 elements per CTA");

  __shared__ Shared<CS> sm;
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
  const int sel = a.select_mode;
  const bool force_radix = (a.flags & MTR_FLAG_FORCE_RADIX) != 0;

  auto id_of = [&](int k) -> int { return base + ((k / VEC) * THREADS + tid) * VEC + (k % VEC); };
  auto chunk_id = [&](int j) -> int { return base + (j * THREADS + tid) * VEC; };

  // ------------------------------------------------------------ prologue
  // this CTA's logits and first history ids are requested before the prologue's
  // dependent-load chains, so their latency overlaps the chains' instead of
  // following it on the warps that run a chain
  const Tin* r1 = (const Tin*)a.logits + row * a.logits_row_stride;
  const Tin* r2 = r1 + dv.second * a.logits_row_stride;
  uint4 ra[NCH], rb[NCH];
  if (dv.vec_ok) {
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int id0 = chunk_id(j);
      ra[j] = make_uint4(0u, 0u, 0u, 0u);
      rb[j] = make_uint4(0u, 0u, 0u, 0u);
      if (id0 < V) {
        ra[j] = __ldcs((const uint4*)(r1 + id0));
        if (a.cfg_enabled) rb[j] = __ldcs((const uint4*)(r2 + id0));
      }
    }
  }
  int64_t hist0 = -1, hist1 = -1;  // first history ids of the penalty window
  if (dv.pen_on) {
    const int i0 = a.penalty_start + tid, i1 = i0 + THREADS;
    if (i0 < L) hist0 = load_id(a, row, i0);
    if (i1 < L) hist1 = load_id(a, row, i1);
  }
  for (int i = tid; i < NB; i += THREADS) sm.hcnt[i] = 0u;
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
      lts = max(lts, __shfl_xor_sync(FULL, lts, o));
      lsos = max(lsos, __shfl_xor_sync(FULL, lsos, o));
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
  // independent dependent-load chains, each on lane 0 of its own warp (lanes of one
  // warp would run the divergent chains one after another): grammar on warp 0,
  // monotonic state on warp 1, conditional temperature on warp 2, uniform on warp 3
  if (lane == 0) {
    if (warp == 1) {
      if (a.mono_mode == MTR_MONO_STATE) {
        mono = a.mono_state[row];
        if ((a.flags & MTR_FLAG_MONO_UPDATE_FROM_IDS) && L > 0) mono = mono_update(a, mono, load_id(a, row, L - 1));
      }
      sm.mono = mono;
      sm.mono_hi = mono >= 0 ? (int32_t)min((int64_t)a.ts_end, (int64_t)a.ts_start + mono) : -1;
    } else if (warp == 0) {
      uint32_t status = 0, allow = 0xffffffffu;
      int gon = 0;
      const uint32_t* gbits = nullptr;
      if (a.grammar_class_of) {
        int64_t prev = -1;
        if (a.flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) prev = L > 0 ? load_id(a, row, L - 1) : -1;
        else if (a.prev_token) prev = a.prev_token[row];
        if (prev >= V) status |= MTR_ROW_BAD_ID;
        if (prev >= 0 && prev < V) {
          const uint32_t c = __ldg(a.grammar_class_of + prev);
          if (c < (uint32_t)a.grammar_n_classes) {
            gon = 1;
            if (a.grammar_vocab_bits) gbits = a.grammar_vocab_bits + (size_t)c * dv.gwords;
            else allow = __ldg(a.grammar_allow + c);  // the class-byte path needs the allow row
          } else {
            status |= MTR_ROW_BAD_ID;
          }
        }
      }
      sm.allow = allow;
      sm.grammar_on = gon;
      sm.gbits = gbits;
      sm.status_g = status;
    } else if (warp == 2) {
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
    } else if (warp == 3) {
      float u = 0.0f;
      uint32_t status = 0;
      if (sel == MTR_SELECT_SAMPLE) {
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
      sm.status_u = status;
    } else if (warp == 5) {
      if (a.lookback_mode == MTR_LOOKBACK_RENORM) {
        int timed = 0;
        if (L > 0) {
          const int64_t t = load_id(a, row, L - 1);
          timed = t >= 0 && t < V && ((__ldg(a.lb_timed_bits + (t >> 5)) >> (t & 31)) & 1u);
        }
        sm.lb_timed = timed;
        sm.lb_p = a.lb_state[row];
      }
    } else if (warp == 6) {
      // first touches of the parameter lines only the epilogue reads: done here,
      // they overlap the prologue instead of missing the constant cache one after
      // another in the row's serial tail
      sm.warm = (uint32_t)a.n_eos_ranges + (uint32_t)a.lookback_mode + (uint32_t)(a.stop_counts != nullptr) +
                (uint32_t)(a.id_buffer != nullptr) + (uint32_t)a.n_eos + (uint32_t)(a.unfinished != nullptr) +
                (uint32_t)(a.out_status != nullptr) + (uint32_t)a.pad_id;
    } else if (warp == 4) {
      sm.status = 0u;
      sm.n_uniq = 0;
      sm.nc = 0;
      sm.nm = 0;
      sm.token = -1;
    }
  }

  // ------------------------------------------------------------ load (+ CFG)
  float x[EPT];
  if (dv.vec_ok) {
    if (a.cfg_enabled) {
      // three separately rounded scalar ops: ptxas rewrites a packed
      // mul.rn.f32x2 -> add.rn.f32x2 chain, which would change the rounding
      const float sc = a.cfg_scale;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float va = E::get(ra[j], e), vb = E::get(rb[j], e);
          x[j * VEC + e] = __fadd_rn(vb, __fmul_rn(__fsub_rn(va, vb), sc));
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < NCH; ++j)
#pragma unroll
        for (int e = 0; e < VEC; ++e) x[j * VEC + e] = E::get(ra[j], e);
    }
  } else {
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const int id = id_of(k);
      float v = 0.0f;
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
  if (warp == 0) {
    // warp 0 stages this CTA's words of the grammar bitmap, so the masks below
    // read shared memory instead of a fourth dependent global load
    __syncwarp();
    const uint32_t* gb = sm.gbits;
    if (gb) {
      const int w0 = base >> 5, nw = min(TILE >> 5, dv.gwords - w0);
      for (int k = lane; k < nw; k += 32) sm.gword[k] = __ldg(gb + w0 + k);
    }
  }
  __syncthreads();  // prologue scalars visible

  // ------------------------------------------------------------ masks (per 8-id chunk)
  {
    const int mono_hi = sm.mono_hi;
    const int ts0 = a.ts_start;
    const bool gon = sm.grammar_on != 0;
    const uint32_t* gbits = sm.gbits;
    const uint32_t allow = sm.allow;
    const uint32_t ncls = (uint32_t)a.grammar_n_classes;
    const bool ragged = (base + TILE) > V;
    if (ragged || mono_hi > ts0 || gon) {
      constexpr uint32_t ALL = (1u << VEC) - 1u;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        const int id0 = chunk_id(j);
        uint32_t keep = range_bits(0, V - id0) & ALL;      // ids < V
        keep &= ~range_bits(ts0 - id0, mono_hi - id0);    // monotonic: [ts0, mono_hi) removed
        if (gon && id0 < V) {
          if (gbits) {
            keep &= sm.gword[(id0 - base) >> 5] >> (id0 & 31);  // id0 % VEC == 0: the chunk sits in one word
          } else {
            uint32_t g = 0;
            if (dv.cls_vec) {
              if constexpr (VEC == 8) {
                const uint2 w = __ldg((const uint2*)(a.grammar_class_of + id0));
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const uint32_t c = ((e < 4 ? w.x : w.y) >> (8 * (e & 3))) & 0xffu;
                  g |= (c < ncls ? (allow >> c) & 1u : 0u) << e;
                }
              } else {
                const uint32_t w = __ldg((const uint32_t*)(a.grammar_class_of + id0));
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  const uint32_t c = (w >> (8 * e)) & 0xffu;
                  g |= (c < ncls ? (allow >> c) & 1u : 0u) << e;
                }
              }
            } else {
#pragma unroll
              for (int e = 0; e < VEC; ++e) {
                if (id0 + e < V) {
                  const uint32_t c = __ldg(a.grammar_class_of + id0 + e);
                  g |= (c < ncls ? (allow >> c) & 1u : 0u) << e;
                }
              }
            }
            keep &= g;
          }
        }
        keep &= ALL;
        if (keep != ALL) {
#pragma unroll
          for (int e = 0; e < VEC; ++e)
            if (!((keep >> e) & 1u)) x[j * VEC + e] = NEG;
        }
      }
    }
    if (a.timeshift_bias != 0.0f) {
      const int ts1 = a.ts_end;
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        const int id = id_of(k);
        if (id >= ts0 && id < ts1) x[k] = __fadd_rn(x[k], a.timeshift_bias);
      }
    }
  }

  // ------------------------------------------------------------ penalties
  if (dv.pen_on) {
    float* xs = (float*)dsm;
    uint32_t* cnt = (uint32_t*)(xs + TILE);
    uint16_t* uniq = (uint16_t*)(cnt + TILE);
    for (int i = tid * 4; i < TILE; i += THREADS * 4) *(uint4*)(cnt + i) = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int li0 = (j * THREADS + tid) * VEC;
#pragma unroll
      for (int e = 0; e < VEC; e += 4)
        *(float4*)(xs + li0 + e) = make_float4(x[j * VEC + e], x[j * VEC + e + 1], x[j * VEC + e + 2], x[j * VEC + e + 3]);
    }
    __syncthreads();
    uint32_t bad = 0;
    for (int i0 = a.penalty_start; i0 < L; i0 += THREADS) {  // block-uniform trip count
      const int i = i0 + tid;
      bool first = false;
      int li = 0;
      if (i < L) {
        const int64_t t = (i0 == a.penalty_start) ? hist0
                          : (i0 == a.penalty_start + THREADS) ? hist1 : load_id(a, row, i);
        if (t < 0 || t >= V) {
          bad = 1;
        } else if (t >= base && t < base + TILE) {
          li = (int)(t - base);
          first = atomicAdd(&cnt[li], 1u) == 0u;
        }
      }
      const unsigned m = __ballot_sync(FULL, first);
      if (m) {
        const int leader = __ffs(m) - 1;
        int slot = 0;
        if (lane == leader) slot = atomicAdd(&sm.n_uniq, __popc(m));
        slot = __shfl_sync(FULL, slot, leader);
        if (first) uniq[slot + __popc(m & ((1u << lane) - 1u))] = (uint16_t)li;
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
    for (int j = 0; j < NCH; ++j) {
      const int id0 = chunk_id(j);
      // the range (first match) of the chunk's first and last id
      float t0 = a.temperature, y0 = dv.temp_rcp, t1 = a.temperature, y1 = dv.temp_rcp;
      for (int r = a.n_col_ranges - 1; r >= 0; --r) {
        if (id0 >= a.col_start[r] && id0 < a.col_end[r]) {
          t0 = a.col_temperature[r];
          y0 = dv.col_rcp[r];
        }
        if (id0 + VEC - 1 >= a.col_start[r] && id0 + VEC - 1 < a.col_end[r]) {
          t1 = a.col_temperature[r];
          y1 = dv.col_rcp[r];
        }
      }
      bool uniform_chunk = t0 == t1;
      if (uniform_chunk) {  // no range edge may split the chunk
        for (int r = 0; r < a.n_col_ranges; ++r) {
          const int s = a.col_start[r], e = a.col_end[r];
          if ((s > id0 && s < id0 + VEC) || (e > id0 && e < id0 + VEC)) uniform_chunk = false;
        }
      }
      if (uniform_chunk) {
        if (t0 != 1.0f) {
          if constexpr (VEC == 8) {
            float v8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v8[e] = x[j * VEC + e];
            div_chunk(v8, t0, y0);
#pragma unroll
            for (int e = 0; e < 8; ++e) x[j * VEC + e] = v8[e];
          } else {
#pragma unroll
            for (int e = 0; e < VEC; e += 2) div_by2(x[j * VEC + e], x[j * VEC + e + 1], t0, y0);
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const int id = id0 + e;
          float t = a.temperature, y = dv.temp_rcp;
          for (int r = a.n_col_ranges - 1; r >= 0; --r) {
            if (id >= a.col_start[r] && id < a.col_end[r]) {
              t = a.col_temperature[r];
              y = dv.col_rcp[r];
            }
          }
          if (t != 1.0f) x[j * VEC + e] = div_by(x[j * VEC + e], t, y);
        }
      }
    }
  } else {
    const float t = sm.t_row, y = sm.t_rcp;
    if (t != 1.0f) {
#pragma unroll
      for (int k = 0; k < EPT; k += 2) div_by2(x[k], x[k + 1], t, y);
    }
  }

  // ------------------------------------------------------------ lookback bias
  // logit_processors.py:143-170.  Mask form: [lb_start, lb_end) -> -inf.
  // Renormalising form: the row's maximum, then the fixed-point masses Q (all
  // finite), O (outside the range) and E (the EOS ids) give the next state E/Q
  // and, after a timed-event token with a known previous state, the shift c
  // (lookback_consts) applied in double to the scores outside the range.
  if (a.lookback_mode == MTR_LOOKBACK_MASK) {
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      const int id = id_of(k);
      if (id >= a.lb_start && id < a.lb_end) x[k] = NEG;
    }
  } else if (a.lookback_mode == MTR_LOOKBACK_RENORM) {
    float m0 = NEG;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < EPT; ++k) {
      bad |= x[k] != x[k] || x[k] == pos_inf();
      m0 = fmaxf(m0, x[k]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m0 = fmaxf(m0, __shfl_xor_sync(FULL, m0, o));
    bad = __any_sync(FULL, bad);
    if (lane == 0) {
      sm.wf[warp] = m0;
      sm.wu2[warp] = bad;
    }
    __syncthreads();
    if (tid == 0) {
      float m = NEG;
      uint32_t b = 0;
      for (int w = 0; w < NW; ++w) {
        m = fmaxf(m, sm.wf[w]);
        b |= sm.wu2[w];
      }
      sm.lbx.mx = m;
      sm.lbx.nan = b;
    }
    Clu<CS>::sync();
    float m = NEG;
    uint32_t rbad = 0;
#pragma unroll
    for (int r = 0; r < CS; ++r) {
      const StatX st = *Clu<CS>::at(&sm.lbx, r);
      m = fmaxf(m, st.mx);
      rbad |= st.nan;
    }
    if (rbad || m == NEG) {  // row-uniform: the row is left as it is
      if (tid == 0) sm.lb_new = __int_as_float(0x7fc00000);
    } else {
      u64 q = 0, o = 0, e = 0;
      const int nle = a.n_lb_eos;
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        if (!(x[k] > NEG)) continue;
        const u64 qv = expfx(__fsub_rn(x[k], m));
        const int id = id_of(k);
        q += qv;
        if (id < a.lb_start || id >= a.lb_end) o += qv;
        for (int j = 0; j < nle; ++j)
          if (a.lb_eos_ids[j] == id) e += qv;
      }
      q = warp_sum_u64(q);
      o = warp_sum_u64(o);
      e = warp_sum_u64(e);
      if (lane == 0) {
        sm.wl[warp * 4 + 0] = q;
        sm.wl[warp * 4 + 1] = o;
        sm.wl[warp * 4 + 2] = e;
      }
      __syncthreads();
      if (tid == 0) {
        u64 t0 = 0, t1 = 0, t2 = 0;
        for (int w = 0; w < NW; ++w) {
          t0 += sm.wl[w * 4 + 0];
          t1 += sm.wl[w * 4 + 1];
          t2 += sm.wl[w * 4 + 2];
        }
        sm.lbs[0] = t0;
        sm.lbs[1] = t1;
        sm.lbs[2] = t2;
      }
      Clu<CS>::sync();
      if (tid == 0) {
        u64 Q = 0, O = 0, Em = 0;
        for (int r = 0; r < CS; ++r) {
          const u64* p = Clu<CS>::at(sm.lbs, r);
          Q += p[0];
          O += p[1];
          Em += p[2];
        }
        sm.lb_new = __double2float_rn(__ddiv_rn((double)Em, (double)Q));
        const float pf = sm.lb_p;
        const int on = sm.lb_timed && pf == pf;
        sm.lb_do = on;
        if (on) lookback_consts(Q, O, pf, m, &sm.lb_c, &sm.lb_v);
      }
      __syncthreads();
      if (sm.lb_do) {
        const double c = sm.lb_c;
        const float lv = sm.lb_v;
#pragma unroll
        for (int k = 0; k < EPT; ++k) {
          const int id = id_of(k);
          if (id >= V) continue;
          if (id == a.lb_start) x[k] = lv;
          else if (id > a.lb_start && id < a.lb_end) x[k] = NEG;
          else x[k] = __double2float_rn(__dsub_rn((double)x[k], c));
        }
      }
    }
  }

  // ------------------------------------------------------------ row statistics
  float lm = NEG;  // this thread's maximum (bound for top-k)
  float gmax;
  int32_t gamax = NO_ID, gnan = NO_ID;
  uint32_t gstatus;
  {
    int32_t la = NO_ID, ln = NO_ID;
    bool nan = false;
    if (sel == MTR_SELECT_ARGMAX) {
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        const float v = x[k];
        if (v != v) ln = min(ln, id_of(k));
        if (v > lm) {
          lm = v;
          la = id_of(k);
        }
      }
      nan = ln != NO_ID;
    } else {
#pragma unroll
      for (int k = 0; k < EPT; ++k) {
        lm = fmaxf(lm, x[k]);
        nan |= x[k] != x[k];
      }
    }
    float wm = lm;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(FULL, wm, o);
      const int32_t oa = __shfl_xor_sync(FULL, la, o);
      if (om > wm || (om == wm && oa < la)) {
        wm = om;
        la = oa;
      }
      ln = min(ln, __shfl_xor_sync(FULL, ln, o));
    }
    const bool wnan = __any_sync(FULL, nan);
    if (lane == 0) {
      sm.wf[warp] = wm;
      sm.wi[warp] = la;
      sm.wi2[warp] = ln;
      sm.wu2[warp] = wnan;
    }
    __syncthreads();
    if (tid == 0) {
      float m = NEG;
      int32_t am = NO_ID, an = NO_ID;
      uint32_t p = 0;
      for (int w = 0; w < NW; ++w) {
        if (sm.wf[w] > m || (sm.wf[w] == m && sm.wi[w] < am)) {
          m = sm.wf[w];
          am = sm.wi[w];
        }
        an = min(an, sm.wi2[w]);
        p |= sm.wu2[w];
      }
      sm.stat.mx = m;
      sm.stat.amax = am;
      sm.stat.nan = p;
      sm.stat.status = sm.status | sm.status_g | sm.status_u;
      sm.red_i[1] = an;
    }
    Clu<CS>::sync();
    gmax = NEG;
    gstatus = 0;
    uint32_t gn = 0;
#pragma unroll
    for (int r = 0; r < CS; ++r) {
      const StatX s = *Clu<CS>::at(&sm.stat, r);
      if (s.mx > gmax || (s.mx == gmax && s.amax < gamax)) {
        gmax = s.mx;
        gamax = s.amax;
      }
      gn |= s.nan;
      gstatus |= s.status;
      if (sel == MTR_SELECT_ARGMAX) gnan = min(gnan, *Clu<CS>::at(&sm.red_i[1], r));
    }
    if (gn && gnan == NO_ID) gnan = NO_ID - 1;  // NaN present (its id only matters for argmax)
  }
  const bool nonfinite = gnan != NO_ID || gmax == pos_inf();
  const bool all_masked = !nonfinite && gmax == NEG;
  if (nonfinite) gstatus |= MTR_ROW_NONFINITE;
  if (all_masked) gstatus |= MTR_ROW_ALL_MASKED;
  const bool clean = !nonfinite && !all_masked;

  // selection state
  float tk = NEG;           // top-k threshold: survivors are finite x >= tk
  bool topk_active = false;
  uint32_t nsurv = 0;       // survivors (valid when topk_active)
  bool list_ready = false;  // the candidate list holds every survivor
  int list_n = 0;
  bool topp_cut = false;    // keep also requires canonical <= (cut_x, cut_id)
  float cut_x = 0.0f;
  int32_t cut_id = NO_ID;
  u64 qkept = 0;
  int32_t token = -1;
  int owner = 0;            // cluster rank that writes the row's scalar outputs
  const float* lx = sm.cx;
  const int32_t* lid = sm.cid;
  uint32_t* lq = sm.cq;
  const bool want_lp = a.out_logprobs != nullptr;
  const bool need_mass = clean && (sel == MTR_SELECT_SAMPLE || want_lp || (sel == MTR_SELECT_NONE && dv.topp_on));
  uint32_t qz[EPT];  // placeholder when collecting without probabilities
#pragma unroll
  for (int k = 0; k < EPT; ++k) qz[k] = 0u;

  // finite-element count of the row (block + cluster)
  auto count_finite = [&]() -> uint32_t {
    uint32_t nf = 0;
#pragma unroll
    for (int k = 0; k < EPT; ++k) nf += finite_val(x[k]);
    nf = warp_sum_u32(nf);
    Clu<CS>::sync();  // wu / cta_nfin free for reuse
    if (lane == 0) sm.wu[warp] = nf;
    __syncthreads();
    if (tid == 0) {
      uint32_t t = 0;
      for (int w = 0; w < NW; ++w) t += sm.wu[w];
      sm.cta_nfin = t;
    }
    Clu<CS>::sync();
    uint32_t t = 0;
#pragma unroll
    for (int r = 0; r < CS; ++r) t += *Clu<CS>::at(&sm.cta_nfin, r);
    return t;
  };

  // merged histogram counts / masses (CS > 1 sums every CTA's bins)
  auto merged_counts = [&](int nbins) -> const uint32_t* {
    if constexpr (CS == 1) {
      return sm.hcnt;
    } else {
      for (int i = tid; i < nbins; i += THREADS) {
        uint32_t c = 0;
#pragma unroll
        for (int r = 0; r < CS; ++r) c += Clu<CS>::at(sm.hcnt, r)[i];
        sm.hcnt_m[i] = c;
      }
      __syncthreads();
      return sm.hcnt_m;
    }
  };
  auto merged_masses = [&](int nbins) -> const u64* {
    if constexpr (CS == 1) {
      return sm.hmass;
    } else {
      for (int i = tid; i < nbins; i += THREADS) {
        u64 m = 0;
#pragma unroll
        for (int r = 0; r < CS; ++r) m += Clu<CS>::at(sm.hmass, r)[i];
        sm.hmass_m[i] = m;
      }
      __syncthreads();
      return sm.hmass_m;
    }
  };

  // radix fallback over this CTA's elements: finds v with W(> v) <= lim <
  // W(>= v) among candidates (pred), descending by key, weights wt; above0 =
  // weight ranked above all candidates.  Returns v, W(> v) and the count /
  // weight of key == v.
  auto radix_select = [&](auto pred, auto keyf, auto wt, u64 lim, u64 above0, uint32_t& out_key, u64& out_above,
                          uint32_t& out_cnt, u64& out_w) {
    uint32_t prefix = 0, mask = 0;
    u64 above = above0;
    u64 lastw = 0;
    uint32_t lastc = 0;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
      Clu<CS>::sync();  // previous readers of the histograms are done
      for (int i = tid; i < 256; i += THREADS) {
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
      const uint32_t* hc = merged_counts(256);
      const u64* hm = merged_masses(256);
      find_crossing<256>(hm, lim - above, &sm.cr);
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

  // merge the per-CTA candidate lists; returns the total (entries stored only
  // when the total fits CAP).  After it every CTA of the cluster holds the
  // same merged list, so list-only stages need no further exchange.
  auto merge_lists = [&]() -> int {
    Clu<CS>::sync();
    if constexpr (CS == 1) {
      lx = sm.cx;
      lid = sm.cid;
      lq = sm.cq;
      return sm.nc;
    } else {
      int tot = 0;
      int offs[CS];
#pragma unroll
      for (int r = 0; r < CS; ++r) {
        offs[r] = tot;
        tot += *Clu<CS>::at(&sm.nc, r);
      }
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
      return tot;
    }
  };

  // start a new local candidate list (after every reader of the previous one)
  auto reset_list = [&]() {
    Clu<CS>::sync();
    if (tid == 0) sm.nc = 0;
    __syncthreads();
  };

  // exact k-th value among n listed values: thread i counts the entries above it
  auto kth_in_list = [&](int n, u64 above, u64 lim) {
    if (tid < n) {
      const float xi = lx[tid];
      uint32_t gt = 0, ge = 0;
      for (int jj = 0; jj < n; ++jj) {
        const float xj = lx[jj];
        gt += xj > xi;
        ge += xj >= xi;
      }
      if (above + gt <= lim && lim < above + ge) {
        sm.tk = xi;
        sm.nsurv = (uint32_t)(above + ge);
      }
    }
    __syncthreads();
  };

  // zero the 1024-entry mass histogram (CTA-local use only)
  auto zero_hmass = [&]() {
    for (int i = tid * 2; i < NB; i += THREADS * 2) *(uint4*)(sm.hmass + i) = make_uint4(0u, 0u, 0u, 0u);
  };

  // entries of the list (index < n) that satisfy `pred` move to the crossing-bin
  // list; returns its size (entries past MINI are counted only)
  auto gather_mini = [&](int n, auto pred) -> int {
    if (tid == 0) sm.nm = 0;
    __syncthreads();
    if (tid < n && pred(tid)) {
      const int s = atomicAdd(&sm.nm, 1);
      if (s < MINI) {
        sm.nx[s] = lx[tid];
        sm.nid[s] = lid[tid];
        sm.nq[s] = lq[tid];
      }
    }
    __syncthreads();
    return sm.nm;
  };

  // ------------------------------------------------------------ selection
  if (clean && sel == MTR_SELECT_ARGMAX) {
    token = gamax;
  } else if (clean) {
    // ---------------- top-k
    if (dv.topk_on) {
      const u64 lim = (u64)(a.top_k - 1);
      bool done = false;
      if (!force_radix) {
        // bound from the per-thread maxima: every thread whose maximum lies in
        // bins <= btau owns at least one element there, so >= k elements do
        if (lm > NEG) atomicAdd(&sm.hcnt[dbin(gmax, lm)], 1u);
        Clu<CS>::sync();
        find_crossing<NB>(merged_counts(NB), lim, &sm.cr);
        const int btau = sm.cr.bin;
        if (btau >= 0) {
          const float c = btau >= NB - 1 ? pos_inf() : (float)(btau + 1) * (1.0f / BIN_SCALE);
          uint32_t mask = 0;
#pragma unroll
          for (int k = 0; k < EPT; ++k) mask |= (uint32_t)(__fsub_rn(gmax, x[k]) < c) << k;
          collect<CS, EPT>(sm, mask, x, qz, false, id_of, lane);
          const int n = merge_lists();
          if (n <= CAP) {
            // second level: count histogram over the listed values
            for (int i = tid; i < NB; i += THREADS) sm.hcnt[i] = 0u;
            __syncthreads();
            if (tid < n) atomicAdd(&sm.hcnt[dbin(gmax, lx[tid])], 1u);
            __syncthreads();
            find_crossing<NB>(sm.hcnt, lim, &sm.cr);
            const int b2 = max(sm.cr.bin, 0);  // n >= k, so a crossing exists
            const u64 above2 = sm.cr.above;
            const int m = gather_mini(n, [&](int i) { return dbin(gmax, lx[i]) == b2; });
            if (m <= MINI) {
              if (tid < m) {
                const float xi = sm.nx[tid];
                uint32_t gt = 0, ge = 0;
                for (int jj = 0; jj < m; ++jj) {
                  const float xj = sm.nx[jj];
                  gt += xj > xi;
                  ge += xj >= xi;
                }
                if (above2 + gt <= lim && lim < above2 + ge) {
                  sm.tk = xi;
                  sm.nsurv = (uint32_t)(above2 + ge);
                }
              }
              __syncthreads();
            } else {
              kth_in_list(n, 0ull, lim);
            }
            tk = sm.tk;
            nsurv = sm.nsurv;
            topk_active = true;
            list_ready = true;
            list_n = n;
            done = true;
          }
        }
      }
      if (!done) {
        const uint32_t nfin = count_finite();
        if ((u64)a.top_k < (u64)nfin) {
          topk_active = true;
          Clu<CS>::sync();
          for (int i = tid; i < NB; i += THREADS) sm.hcnt[i] = 0u;
          __syncthreads();
#pragma unroll
          for (int k = 0; k < EPT; ++k)
            if (finite_val(x[k])) atomicAdd(&sm.hcnt[dbin(gmax, x[k])], 1u);
          Clu<CS>::sync();
          find_crossing<NB>(merged_counts(NB), lim, &sm.cr);
          const int bstar = max(sm.cr.bin, 0);  // k - 1 < finite count, so a crossing exists
          const u64 c_above = sm.cr.above;
          const u64 n_c = sm.cr.w;
          if (n_c <= (u64)CAP && !force_radix) {
            reset_list();
            uint32_t mask = 0;
#pragma unroll
            for (int k = 0; k < EPT; ++k) mask |= (uint32_t)(finite_val(x[k]) && dbin(gmax, x[k]) == bstar) << k;
            collect<CS, EPT>(sm, mask, x, qz, false, id_of, lane);
            const int n = merge_lists();
            kth_in_list(n, c_above, lim);
            tk = sm.tk;
            nsurv = sm.nsurv;
          } else {
            uint32_t key, cntv;
            u64 abv, wv;
            radix_select([&](int k) { return finite_val(x[k]) && dbin(gmax, x[k]) == bstar; },
                         [&](int k) { return fkey(x[k]); }, [&](int) { return 1u; }, lim, c_above, key, abv, cntv,
                         wv);
            tk = key2f(key);
            nsurv = (uint32_t)(abv + wv);
            gstatus |= MTR_ROW_SLOW_PATH;
          }
        } else {
          nsurv = nfin;  // fewer than k finite scores: top-k removes nothing
        }
      }
    }

    // ---------------- top-p and the draw
    if (need_mass) {
      const bool topp_on = dv.topp_on != 0;
      const float u = sm.u;
      if (topk_active && nsurv <= (uint32_t)CAP && !force_radix) {
        // compact path: every survivor is in the list; other entries get q = 0
        if (!list_ready) {
          reset_list();
          uint32_t mask = 0;
#pragma unroll
          for (int k = 0; k < EPT; ++k) mask |= (uint32_t)(finite_val(x[k]) && x[k] >= tk) << k;
          collect<CS, EPT>(sm, mask, x, qz, false, id_of, lane);
          list_n = merge_lists();
        }
        const int n = list_n;
        float xi = 0.0f;
        int32_t ii = 0;
        uint32_t qi = 0;
        if (tid < n) {
          xi = lx[tid];
          ii = lid[tid];
          qi = xi >= tk ? expfx(__fsub_rn(xi, gmax)) : 0u;
          lq[tid] = qi;
        }
        // total mass
        {
          const u64 s = warp_sum_u64((u64)qi);
          if (lane == 0) sm.wl[warp] = s;
          zero_hmass();
          __syncthreads();
          u64 t = 0;
#pragma unroll
          for (int w = 0; w < NW; ++w) t += sm.wl[w];
          qkept = t;
        }
        const u64 tot = qkept;
        if (topp_on) {
          const double P = __dmul_rn((double)a.top_p, (double)tot);
          const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
          if (qi) atomicAdd(&sm.hmass[dbin(gmax, xi)], (u64)qi);
          __syncthreads();
          find_crossing<NB>(sm.hmass, plim, &sm.cr);
          const int b3 = max(sm.cr.bin, 0);  // plim < total
          const u64 above3 = sm.cr.above;
          const int m = gather_mini(n, [&](int i) { return lq[i] != 0u && dbin(gmax, lx[i]) == b3; });
          if (m <= MINI) {
            if (tid < m) {
              const float xm = sm.nx[tid];
              const int32_t im = sm.nid[tid];
              const u64 qm = sm.nq[tid];
              u64 am = above3;
              for (int jj = 0; jj < m; ++jj)
                if (canon_before(sm.nx[jj], sm.nid[jj], xm, im)) am += sm.nq[jj];
              if (am <= plim && am + qm > plim) {
                sm.cut_x = xm;
                sm.cut_id = im;
                sm.qkept = am + qm;
              }
            }
          } else if (tid < n && qi) {
            u64 ai = 0;
            for (int jj = 0; jj < n; ++jj)
              if (canon_before(lx[jj], lid[jj], xi, ii)) ai += lq[jj];
            if (ai <= plim && ai + qi > plim) {
              sm.cut_x = xi;
              sm.cut_id = ii;
              sm.qkept = ai + qi;
            }
          }
          __syncthreads();
          topp_cut = true;
          cut_x = sm.cut_x;
          cut_id = sm.cut_id;
          qkept = sm.qkept;
        }
        const bool kept = qi != 0u && (!topp_cut || xi > cut_x || (xi == cut_x && ii <= cut_id));
        if (topp_cut) {
          const bool tie = tid < n && xi >= tk && xi == cut_x && ii > cut_id;
          if (__syncthreads_or(tie)) gstatus |= MTR_ROW_TIE_AT_CUT;
        }
        if (sel == MTR_SELECT_SAMPLE) {
          // id-binned kept mass, then the exact draw inside the crossing id bin
          const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
          zero_hmass();
          if (tid < CAP) sm.ckeep[tid] = kept ? 1 : 0;
          __syncthreads();
          if (kept) atomicAdd(&sm.hmass[ii >> dv.id_shift], (u64)qi);
          __syncthreads();
          find_crossing<NB>(sm.hmass, R, &sm.cr);
          const int b4 = max(sm.cr.bin, 0);  // R < qkept
          const u64 above4 = sm.cr.above;
          const int m = gather_mini(n, [&](int i) { return sm.ckeep[i] && (lid[i] >> dv.id_shift) == b4; });
          if (m <= MINI) {
            if (tid < m) {
              const int32_t im = sm.nid[tid];
              const u64 qm = sm.nq[tid];
              u64 cm = above4;
              for (int jj = 0; jj < m; ++jj)
                if (sm.nid[jj] <= im) cm += sm.nq[jj];
              if (cm > R && cm - qm <= R) sm.token = im;
            }
          } else if (kept) {
            u64 ci = 0;
            for (int jj = 0; jj < n; ++jj)
              if (sm.ckeep[jj] && lid[jj] <= ii) ci += lq[jj];
            if (ci > R && ci - qi <= R) sm.token = ii;
          }
          __syncthreads();
          token = sm.token;
        }
      } else {
        // dense path: per-element fixed-point probabilities of the survivors
        uint32_t q[EPT];
#pragma unroll
        for (int k = 0; k < EPT; k += 2) {
          expfx2(__fsub_rn(x[k], gmax), __fsub_rn(x[k + 1], gmax), q[k], q[k + 1]);
          if (!(x[k] >= tk)) q[k] = 0u;
          if (!(x[k + 1] >= tk)) q[k + 1] = 0u;
        }
        if (topp_on) {
          Clu<CS>::sync();
          zero_hmass();
          if (tid == 0) sm.nc = 0;
          __syncthreads();
          // mass histogram as two u32 halves (low / high 16 bits of q): native
          // 32-bit shared atomics, exact for a CTA's <= 2^14 elements
          uint32_t* hlo = (uint32_t*)sm.hmass;
          uint32_t* hhi = hlo + NB;
#pragma unroll
          for (int k = 0; k < EPT; ++k) {
            if (q[k]) {
              const int b = dbin(gmax, x[k]);
              atomicAdd(hlo + b, q[k] & 0xffffu);
              atomicAdd(hhi + b, q[k] >> 16);
            }
          }
          Clu<CS>::sync();
          // total, the limit it implies, and the crossing of the limit, in one pass
          if constexpr (CS == 1) {
            find_topp_crossing_blk<NB, THREADS>([&](int i) -> u64 { return (u64)hlo[i] + ((u64)hhi[i] << 16); },
                                                a.top_p, a.top_p_mode, &sm.cr, &sm.plim, sm.wl);
          } else {
            for (int i = tid; i < NB; i += THREADS) {
              u64 m = 0;
#pragma unroll
              for (int r = 0; r < CS; ++r) {
                const uint32_t* rl = (const uint32_t*)Clu<CS>::at(sm.hmass, r);
                m += (u64)rl[i] + ((u64)rl[NB + i] << 16);
              }
              sm.hmass_m[i] = m;
            }
            __syncthreads();
            find_topp_crossing<NB>([&](int i) -> u64 { return sm.hmass_m[i]; }, a.top_p, a.top_p_mode, &sm.cr,
                                   &sm.plim);
          }
          const u64 plim = sm.plim;
          const int bstar = max(sm.cr.bin, 0);  // plim < total since top_p < 1
          const u64 w_above = sm.cr.above;
          const float lo = (float)bstar * (1.0f / BIN_SCALE), hi = (float)(bstar + 1) * (1.0f / BIN_SCALE);
          uint32_t mask = 0;
#pragma unroll
          for (int k = 0; k < EPT; ++k) {
            const float d = __fsub_rn(gmax, x[k]);
            mask |= (uint32_t)(q[k] != 0u && d >= lo && (bstar >= NB - 1 || d < hi)) << k;
          }
          collect<CS, EPT>(sm, mask, x, q, true, id_of, lane);
          const int n = merge_lists();
          if (n <= CAP && !force_radix) {
            if (n <= 32) {
              // one warp: lane j holds candidate j and sums the mass canonically before it
              if (warp == 0) {
                const float xj = lane < n ? lx[lane] : 0.0f;
                const int32_t ij = lane < n ? lid[lane] : NO_ID;
                const uint32_t qj = lane < n ? lq[lane] : 0u;
                u64 aj = w_above;
#pragma unroll 4
                for (int i = 0; i < n; ++i) {
                  const float xi = __shfl_sync(FULL, xj, i);
                  const int32_t ii = __shfl_sync(FULL, ij, i);
                  const uint32_t qi = __shfl_sync(FULL, qj, i);
                  aj += canon_before(xi, ii, xj, ij) ? (u64)qi : 0ull;
                }
                if (lane < n && aj <= plim && aj + qj > plim) {
                  sm.cut_x = xj;
                  sm.cut_id = ij;
                  sm.qkept = aj + qj;
                }
              }
            } else if (tid < n) {
              const float xi = lx[tid];
              const int32_t ii = lid[tid];
              const u64 qi = lq[tid];
              u64 ai = w_above;
              for (int jj = 0; jj < n; ++jj)
                if (canon_before(lx[jj], lid[jj], xi, ii)) ai += lq[jj];
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
            const bool tie = tid < n && lx[tid] == cut_x && lid[tid] > cut_id;
            if (__syncthreads_or(tie)) gstatus |= MTR_ROW_TIE_AT_CUT;
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
        // drop the removed tail from q (kept = survivors up to the cut)
        if (topp_cut) {
#pragma unroll
          for (int k = 0; k < EPT; ++k) {
            const float v = x[k];
            if (!(v > cut_x || (v == cut_x && id_of(k) <= cut_id))) q[k] = 0u;
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
          if constexpr (CS == 1) {
            // ids run chunk-major (chunk j of every thread, then chunk j + 1), so one
            // warp scan per chunk and the warp totals locate the thread and chunk
            // holding the draw without forming the CTA total first
            if (tid == 0) sm.token = 0;
            __syncthreads();  // wl free for reuse
            u64 inc[NCH];
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
              inc[j] = warp_incl_scan_u64(cs[j], lane);
              if (lane == 31) sm.wl[j * 32 + warp] = inc[j];
            }
            __syncthreads();
            u64 chunk_base = 0;
#pragma unroll
            for (int j = 0; j < NCH; ++j) {
              u64 wb = 0, wt = 0;
              for (int w = 0; w < NW; ++w) {
                const u64 v = sm.wl[j * 32 + w];
                wb += w < warp ? v : 0ull;
                wt += v;
              }
              const u64 lo = chunk_base + wb + inc[j] - cs[j];
              if (cs[j] != 0 && lo <= R && R < lo + cs[j]) {
                u64 c = lo;
                bool found = false;
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  c += q[j * VEC + e];
                  if (!found && c > R) {
                    sm.token = id_of(j * VEC + e);
                    found = true;
                  }
                }
              }
              chunk_base += wt;
            }
            __syncthreads();
            token = sm.token;
          } else {
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
                bool found = false;
  #pragma unroll
                for (int j = 0; j < NCH; ++j) {
  #pragma unroll
                  for (int e = 0; e < VEC; ++e) {
                    const int k = j * VEC + e;
                    if (j == jstar && !found) {
                      c += q[k];
                      if (c > rr) {
                        sm.token = id_of(k);
                        found = true;
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
  }
  if (!clean && sel == MTR_SELECT_ARGMAX) token = gnan != NO_ID ? gnan : (gmax == NEG ? 0 : gamax);
  if (!clean && sel == MTR_SELECT_SAMPLE) token = (int32_t)a.pad_id;

  // ------------------------------------------------------------ epilogue
  // processed scores: survivors of top-k and top-p; unfiltered for argmax
  const bool filter_out = clean && sel != MTR_SELECT_ARGMAX;
  auto kept_at = [&](float v, int id) -> bool {
    if (!(v >= tk)) return false;
    return !topp_cut || v > cut_x || (v == cut_x && id <= cut_id);
  };
  if (a.out_scores) {
    float* orow = a.out_scores + row * a.out_scores_row_stride;
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int id0 = chunk_id(j);
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float v = x[j * VEC + e];
        o[e] = (filter_out && !kept_at(v, id0 + e)) ? NEG : v;
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
      const int id0 = chunk_id(j);
      float o[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        const float v = x[j * VEC + e];
        bool kp = finite_val(v);
        if (filter_out) kp = kp && kept_at(v, id0 + e);
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
      const int64_t fin = finish_token(a, row, token, &gstatus);
      if (a.flags & MTR_FLAG_MONO_UPDATE_FROM_SAMPLE) m = mono_update(a, m, fin);
      if ((a.flags & MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE) && a.prev_token) a.prev_token[row] = (int32_t)fin;
      if (a.out_ids) a.out_ids[row] = fin;
    }
    if (a.mono_mode != MTR_MONO_OFF && a.mono_state) a.mono_state[row] = m;
    if (a.lookback_mode == MTR_LOOKBACK_RENORM) a.lb_state[row] = sm.lb_new;
    if (a.out_status) a.out_status[row] = gstatus;
  }
  if constexpr (CS > 1) cg::this_cluster().sync();  // no CTA leaves while its shared memory may be read
}

// ---------------------------------------------------------------------------
// row-per-warp kernel: many rows of a vocabulary <= 4096
//
// One warp owns one row at a time and walks rows r, r + grid, ... (persistent
// grid sized by occupancy).  The row's logits arrive in shared memory by bulk
// asynchronous copies (cp.async.bulk, completion on an mbarrier) and are
// processed in place into the fp32 row X; the next row's copy is issued as soon
// as X is no longer needed (normally right after the top-k survivors are
// listed), so it lands while the current row finishes its top-p and draw.  No
// block barrier exists: cross-lane steps are shuffles, ballots and __syncwarp.
//
// X layout.  16-bit logits: chunk c (ids 8c .. 8c+7) keeps ids 8c..8c+3 at
// floats [4c, 4c+4) and ids 8c+4..8c+7 at [VP/2 + 4c, ...).  The raw first-half
// row is copied to bytes [0, 2V) and the raw second-half row to [2VP, 2VP+2V),
// so chunk c's raw data sits exactly where its processed floats go.  fp32
// logits: natural layout (id i at float i), the raw row copied in place.
//
// Dynamic shared memory per warp: X (VP floats) + a region that holds the
// history counts during the chain and the selection state after it: 16 KB +
// 5504 B at V = 4096, so ten warps fit on an SM (228 KB; per CTA 1 KB reserved,
// 16 B static, 128 B granularity).
// The counts are 8-bit; a row whose window repeats an id 256 times or more, or
// whose penalty window reaches past the ids held in registers, is counted again
// exactly with 16-bit counts over one half of the vocabulary at a time.
// ---------------------------------------------------------------------------
constexpr int WV_MAX = 4096;
constexpr int WNB = 256;               // histogram bins
constexpr float WBIN_SCALE = 8.0f;     // chunk-maximum bins per logit
constexpr int WCAP = 224;              // candidate / survivor list (a multiple of 32)
constexpr int WMINI = 64;              // crossing-bin list
constexpr int WHIST = 16;              // history ids per lane held in registers
constexpr int WSEL_BYTES = WNB * 8 + WCAP * 12 + WMINI * 12;
constexpr int WMAX_PEN_IDS = 32767;    // counts keep a claim bit in bit 15
constexpr uint32_t WAIT_POLLS = 1u << 20;  // ~1 s of 1 us suspends before a copy counts as lost

__host__ __device__ constexpr int warp_vpad(int V) { return (V + 255) / 256 * 256; }
__host__ __device__ constexpr int warp_union_bytes(int V) {
  return warp_vpad(V) > WSEL_BYTES ? warp_vpad(V) : WSEL_BYTES;
}
__host__ __device__ constexpr int warp_bytes(int V) { return warp_vpad(V) * 4 + warp_union_bytes(V); }

__device__ __forceinline__ int wbin(float mx, float x) {
  float s = __fmul_rn(__fsub_rn(mx, x), WBIN_SCALE);
  s = fminf(s, (float)(WNB - 1));
  return __float2int_rz(s);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* m) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(m)) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* m, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(m)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* m, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(m)), "r"(parity), "r"(1000u)
      : "memory");
  return ok != 0;
}
// bounded wait for phase `parity`; false when the copy did not land within
// `polls` polls
__device__ __forceinline__ bool mbar_wait(uint64_t* m, uint32_t parity, uint32_t polls = WAIT_POLLS) {
#pragma unroll 1
  for (uint32_t i = 0; i < polls; ++i)
    if (mbar_try_wait(m, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* m) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(m))
               : "memory");
}
// order this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk copy) writes to it
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Crossing of `lim` in a 256-bin histogram h (lane owns bins 8*lane .. 8*lane+7):
// the bin b with W(bins < b) <= lim < W(bins <= b).  Returns -1 when lim >= total.
template <typename W>
__device__ __forceinline__ int warp_crossing(const W* h, u64 lim, int lane, u64& above, u64& w) {
  W v[8];
  if constexpr (sizeof(W) == 4) {
    const uint4 p0 = *(const uint4*)(h + lane * 8), p1 = *(const uint4*)(h + lane * 8 + 4);
    v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
    v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
  } else {
#pragma unroll
    for (int r = 0; r < 8; r += 2) {
      const ulonglong2 p = *(const ulonglong2*)(h + lane * 8 + r);
      v[r] = p.x;
      v[r + 1] = p.y;
    }
  }
  u64 s = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) s += v[r];
  const u64 incl = warp_incl_scan_u64(s, lane);
  int my_b = -1;
  u64 my_above = 0, my_w = 0;
  if (incl - s <= lim && lim < incl) {
    u64 c = incl - s;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (my_b < 0 && c + v[r] > lim) {
        my_b = lane * 8 + r;
        my_above = c;
        my_w = v[r];
      }
      c += v[r];
    }
  }
  const unsigned bal = __ballot_sync(FULL, my_b >= 0);
  if (!bal) return -1;
  const int src = __ffs(bal) - 1;
  above = __shfl_sync(FULL, my_above, src);
  w = __shfl_sync(FULL, my_w, src);
  return __shfl_sync(FULL, my_b, src);
}

// warp_crossing over a histogram kept as low / high 16-bit sums of its weights
// (bin i weighs lo[i] + hi[i] * 2^16), so its updates are 32-bit shared atomics
__device__ __forceinline__ int warp_crossing_halves(const uint32_t* lo, const uint32_t* hi, u64 lim, int lane,
                                                    u64& above, u64& w) {
  u64 v[8];
  {
    const uint4 l0 = *(const uint4*)(lo + lane * 8), l1 = *(const uint4*)(lo + lane * 8 + 4);
    const uint4 h0 = *(const uint4*)(hi + lane * 8), h1 = *(const uint4*)(hi + lane * 8 + 4);
    v[0] = l0.x + ((u64)h0.x << 16); v[1] = l0.y + ((u64)h0.y << 16);
    v[2] = l0.z + ((u64)h0.z << 16); v[3] = l0.w + ((u64)h0.w << 16);
    v[4] = l1.x + ((u64)h1.x << 16); v[5] = l1.y + ((u64)h1.y << 16);
    v[6] = l1.z + ((u64)h1.z << 16); v[7] = l1.w + ((u64)h1.w << 16);
  }
  u64 s = 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) s += v[r];
  const u64 incl = warp_incl_scan_u64(s, lane);
  int my_b = -1;
  u64 my_above = 0, my_w = 0;
  if (incl - s <= lim && lim < incl) {
    u64 c = incl - s;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (my_b < 0 && c + v[r] > lim) {
        my_b = lane * 8 + r;
        my_above = c;
        my_w = v[r];
      }
      c += v[r];
    }
  }
  const unsigned bal = __ballot_sync(FULL, my_b >= 0);
  if (!bal) return -1;
  const int src = __ffs(bal) - 1;
  above = __shfl_sync(FULL, my_above, src);
  w = __shfl_sync(FULL, my_w, src);
  return __shfl_sync(FULL, my_b, src);
}

// a chunk that a column-range edge splits: element by element (out of line)
__device__ __noinline__ void temp_chunk_split(const MtrSamplerArgs& a, const Derived& dv, float (&v)[8], int id0) {
  for (int e = 0; e < 8; ++e) {
    float te = a.temperature, ye = dv.temp_rcp;
#pragma unroll 1
    for (int r = a.n_col_ranges - 1; r >= 0; --r)
      if (id0 + e >= a.col_start[r] && id0 + e < a.col_end[r]) {
        te = a.col_temperature[r];
        ye = dv.col_rcp[r];
      }
    if (te != 1.0f) v[e] = div_by(v[e], te, ye);
  }
}

// temperature of a chunk: the row's (scalar / conditional) or the column ranges'
// (first match wins; a chunk split by a range edge goes element by element)
__device__ __forceinline__ void temp_chunk(const MtrSamplerArgs& a, const Derived& dv, float (&v)[8], int id0,
                                           float t_row, float y_row) {
  if (a.temp_mode != MTR_TEMP_COLUMN_RANGES) {
    if (t_row != 1.0f) div_chunk(v, t_row, y_row);
    return;
  }
  float t0 = a.temperature, y0 = dv.temp_rcp, t1 = a.temperature;
  bool uniform_chunk = true;
#pragma unroll 1
  for (int r = a.n_col_ranges - 1; r >= 0; --r) {
    const int cs = a.col_start[r], ce = a.col_end[r];
    if (id0 >= cs && id0 < ce) {
      t0 = a.col_temperature[r];
      y0 = dv.col_rcp[r];
    }
    if (id0 + 7 >= cs && id0 + 7 < ce) t1 = a.col_temperature[r];
    if ((cs > id0 && cs < id0 + 8) || (ce > id0 && ce < id0 + 8)) uniform_chunk = false;
  }
  if (uniform_chunk && t0 == t1) {
    if (t0 != 1.0f) div_chunk(v, t0, y0);
    return;
  }
  temp_chunk_split(a, dv, v, id0);
}

// Penalties of up to eight owned window ids (bit k of own8: id ids.t[k]) with
// the IEEE divide for rare operands (zero, tiny, huge or NaN scores, or a
// repetition penalty outside the fast divide's range): the same steps as the
// common loop, out of line so that loop stays short.
struct PenIds8 {
  int32_t t[8];
};
__device__ __noinline__ void pen_rare8(float* X, const uint32_t* cnt, const PenIds8 ids, uint32_t own8, int half,
                                       bool split, float rp, float fp, float pp, float y) {
#pragma unroll 1
  for (int k = 0; k < 8; ++k) {
    if (!((own8 >> k) & 1u)) continue;
    const int t = ids.t[k];
    const int xo = split ? ((t & 4) ? half : 0) + ((t >> 3) << 2) + (t & 3) : t;
    const float c = (float)((cnt[t >> 2] >> (8 * (t & 3))) & 0xffu);
    X[xo] = pen_value(X[xo], c, rp, fp, pp, y);
  }
}
// Penalties from exact 16-bit counts, for rows whose penalty window reaches
// past the ids held in registers or repeats an id 256 times or more: one half
// of the vocabulary at a time, the ids read again, bit 15 of a count claiming
// the id for the lane that applies it.  Out of line: rare rows only.
__device__ __noinline__ void pen_exact(float* X, uint32_t* cnt, const MtrSamplerArgs& a, int64_t row, int L, int V,
                                       int VP, bool split, int lane, float rp, float fp, float pp, float y) {
  const int H = VP / 2;
#pragma unroll 1
  for (int lo = 0; lo < VP; lo += H) {
    __syncwarp();
#pragma unroll 1
    for (int w = lane * 4; w < H / 2; w += 128) *(uint4*)(cnt + w) = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
#pragma unroll 1
    for (int pos = a.penalty_start + lane; pos < L; pos += 32) {
      const int64_t t = load_id(a, row, pos);
      if (t >= lo && t < lo + H && t < V) atomicAdd(cnt + ((t - lo) >> 1), 1u << (16 * ((t - lo) & 1)));
    }
    __syncwarp();
#pragma unroll 1
    for (int pos = a.penalty_start + lane; pos < L; pos += 32) {
      const int64_t t = load_id(a, row, pos);
      if (t >= lo && t < lo + H && t < V) {
        const int r = (int)(t - lo);
        const uint32_t sh = 16u * (uint32_t)(r & 1);
        const uint32_t old = atomicOr(cnt + (r >> 1), 0x8000u << sh);
        if (!((old >> sh) & 0x8000u)) {
          const int ti = (int)t;
          const int xo = split ? ((ti & 4) ? H : 0) + ((ti >> 3) << 2) + (ti & 3) : ti;
          X[xo] = pen_value(X[xo], (float)((old >> sh) & 0x7fffu), rp, fp, pp, y);
        }
      }
    }
  }
  __syncwarp();
}
// per-row values loaded one row ahead.  Loads only: every value stays raw
// (no arithmetic on a loaded register) until the row that uses it, so issuing
// them never waits on memory.
struct WarpAhead {
  u64 hid[WHIST];  // raw ids at positions hbase + lane + 32k (int32 ids zero-extended)
  int32_t hbase;
  // per-row scalars, each loaded straight into its own register (a conversion
  // right after the load would wait for it)
  int32_t mono;    // lane 0: mono_state[row]
  int32_t prev;    // lane 1: prev_token[row]
  uint32_t ubits;  // lane 3: uniforms[row]
  uint32_t last32; // lane 0 / 1: input_ids[row, L - 1] (int32 ids)
  u64 last64;      // lane 0 / 1: input_ids[row, L - 1] (int64 ids)
  uint32_t cond32[MTR_MAX_COND_TEMPS];  // lane 2: input_ids[row, L - cond_offset[c]] (int32 ids)
  u64 cond64[MTR_MAX_COND_TEMPS];       // lane 2: the same (int64 ids)
  uint32_t cls;    // lane 1: grammar class of the previous token, looked up one row ahead
};
constexpr u64 RAW_NONE = 0x8000000000000000ull;  // an id that lies outside int32: never valid

__device__ __forceinline__ int64_t raw_id(const MtrSamplerArgs& a, u64 raw) {
  return a.ids_dtype == MTR_IDS_I32 ? (int64_t)(int32_t)(uint32_t)raw : (int64_t)raw;
}
// as int32 (INT32_MIN when the id does not fit)
__device__ __forceinline__ int32_t narrow_raw(const MtrSamplerArgs& a, u64 raw) {
  const int64_t t = raw_id(a, raw);
  return (t >= INT32_MIN && t <= INT32_MAX) ? (int32_t)t : INT32_MIN;
}

// the previous token of the row ahead (lane 1; -1: none)
// the last id of the row ahead, as int64 (-1 when the history is empty)
__device__ __forceinline__ int64_t ahead_last(const MtrSamplerArgs& a, const WarpAhead& w, int L) {
  if (L <= 0) return -1;
  return a.ids_dtype == MTR_IDS_I32 ? (int64_t)(int32_t)w.last32 : (int64_t)w.last64;
}
// the previous token of the row ahead (lane 1; -1: none)
__device__ __forceinline__ int64_t ahead_prev(const MtrSamplerArgs& a, const WarpAhead& w, int L) {
  if (a.flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) return ahead_last(a, w, L);
  return a.prev_token ? (int64_t)w.prev : -1;
}
// second step of the row-ahead loads, issued once the first step has landed:
// the class of the previous token (lane 1), so the row's prologue has no
// dependent global load on the grammar path
__device__ __forceinline__ void load_ahead_class(const MtrSamplerArgs& a, int lane, int V, int L, WarpAhead& w) {
  w.cls = 0xffffffffu;
  if (lane == 1 && a.grammar_class_of) {
    const int64_t prev = ahead_prev(a, w, L);
    if (prev >= 0 && prev < V) w.cls = __ldg(a.grammar_class_of + prev);
  }
}

__device__ __forceinline__ void load_ahead(const MtrSamplerArgs& a, const Derived& dv, int64_t row, int lane, int L,
                                           WarpAhead& w) {
  w.hbase = L > WHIST * 32 ? L - WHIST * 32 : 0;
#pragma unroll
  for (int k = 0; k < WHIST; ++k) w.hid[k] = RAW_NONE;
  if (dv.pen_on || a.mono_mode == MTR_MONO_SCAN) {
    const int n = L - w.hbase - lane;  // this lane's positions: hbase + lane + 32 k < L
    if (a.ids_dtype == MTR_IDS_I32) {
      const uint32_t* p = (const uint32_t*)a.input_ids + row * a.ids_row_stride + w.hbase + lane;
#pragma unroll
      for (int k = 0; k < WHIST; ++k)
        if (32 * k < n) w.hid[k] = (u64)__ldg(p + 32 * k);
    } else {
      const unsigned long long* p = (const unsigned long long*)a.input_ids + row * a.ids_row_stride + w.hbase + lane;
#pragma unroll
      for (int k = 0; k < WHIST; ++k)
        if (32 * k < n) w.hid[k] = (u64)__ldg(p + 32 * k);
    }
  }
  const bool i32 = a.ids_dtype == MTR_IDS_I32;
  const int64_t roff = row * a.ids_row_stride;
  const bool need_last = L > 0 && ((lane == 0 && (a.flags & MTR_FLAG_MONO_UPDATE_FROM_IDS)) ||
                                   (lane == 1 && a.grammar_class_of && (a.flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS)));
  if (need_last) {
    if (i32) w.last32 = __ldg((const uint32_t*)a.input_ids + roff + L - 1);
    else w.last64 = __ldg((const unsigned long long*)a.input_ids + roff + L - 1);
  }
  if (lane == 0 && a.mono_mode == MTR_MONO_STATE) w.mono = a.mono_state[row];
  if (lane == 1 && a.grammar_class_of && !(a.flags & MTR_FLAG_GRAMMAR_PREV_FROM_IDS) && a.prev_token)
    w.prev = a.prev_token[row];
  if (lane == 3 && a.select_mode == MTR_SELECT_SAMPLE) w.ubits = __float_as_uint(a.uniforms[row]);
  if (lane == 2 && a.temp_mode == MTR_TEMP_ROW_CONDITIONAL) {
#pragma unroll
    for (int c = 0; c < MTR_MAX_COND_TEMPS; ++c) {
      const int off = a.cond_offset[c];
      if (c < a.n_cond && off >= 1 && L >= off) {
        if (i32) w.cond32[c] = __ldg((const uint32_t*)a.input_ids + roff + L - off);
        else w.cond64[c] = __ldg((const unsigned long long*)a.input_ids + roff + L - off);
      }
    }
  }
}

// Result of the row-per-warp kernel's dense mass path.
struct WDense {
  float cut_x;
  int32_t cut_id;
  u64 qkept;
  int32_t token;
  uint32_t status;
  int32_t topp_cut;
  int32_t ok;  // 0: a crossing bin still held more than WMINI candidates after refinement
};

// Top-p and the draw over every score of a staged row when there is no
// survivor list (no top-k, or more survivors than the list holds).  Pass A
// computes the fixed-point mass q of every score >= tk and, with top-p, adds it
// to a histogram of the distance to the max in 1/16-logit bins (monotone in the
// score, so bins follow canonical order); warp_crossing_halves finds the bin
// holding the limit.  Its candidates are listed (a second 256-bin level splits
// the bin when it holds more than WMINI) and resolved in canonical order (score
// descending, id ascending).  The draw walks the 16 id slots of 256 ids in id
// order, one warp scan of the kept masses per slot, and stops in the slot that
// crosses floor(u * Q_kept).  X holds the row as the kernel stages it: chunk c
// (ids 8c .. 8c+7) at lo(c) and hi(c).
template <bool SPLIT>
__device__ __noinline__ void warp_dense(const float* X, int HALF, int nch, int V, float gmax, float tk, bool topp_on,
                                        float top_p, int top_p_mode, bool sample, float u, uint32_t* hlo, float* mx,
                                        int32_t* mi, uint32_t* mq, int lane, WDense* out) {
  constexpr int NS = WV_MAX / 256;
  uint32_t* const hhi = hlo + WNB;
  auto lo_of = [&](int c) -> const float* { return X + (SPLIT ? 4 * c : 8 * c); };
  auto hi_of = [&](int c) -> const float* { return X + (SPLIT ? HALF + 4 * c : 8 * c + 4); };
  auto load8 = [&](int c, float (&v)[8]) {
    const float4 f0 = *(const float4*)lo_of(c), f1 = *(const float4*)hi_of(c);
    v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
    v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
  };
  // fixed-point masses of chunk c's scores that take part (finite, >= tk, id < V)
  auto mass8 = [&](int c, const float (&v)[8], uint32_t (&q)[8]) {
#pragma unroll
    for (int e = 0; e < 8; e += 2) expfx2(__fsub_rn(v[e], gmax), __fsub_rn(v[e + 1], gmax), q[e], q[e + 1]);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (!(finite_val(v[e]) && v[e] >= tk) || 8 * c + e >= V) q[e] = 0u;
  };
  auto bin1 = [&](float x) -> int {
    return __float2int_rz(fminf(__fmul_rn(__fsub_rn(gmax, x), 16.0f), (float)(WNB - 1)));
  };
  auto zero_hist = [&]() {
#pragma unroll
    for (int i = lane * 4; i < 2 * WNB; i += 128) *(uint4*)(hlo + i) = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
  };
  out->ok = 1;
  out->status = 0;
  out->topp_cut = 0;
  out->cut_x = 0.0f;
  out->cut_id = NO_ID;
  out->token = -1;

  // ---- pass A: total mass (and the level-1 histogram)
  if (topp_on) zero_hist();
  u64 tot = 0;
#pragma unroll 1
  for (int s = 0; s < NS; ++s) {
    const int c = s * 32 + lane;
    if (c >= nch) break;
    float v[8];
    uint32_t q[8];
    load8(c, v);
    mass8(c, v, q);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      tot += q[e];
      if (topp_on && q[e]) {
        const int b = bin1(v[e]);
        atomicAdd(hlo + b, q[e] & 0xffffu);
        atomicAdd(hhi + b, q[e] >> 16);
      }
    }
  }
  tot = warp_sum_u64(tot);
  u64 qkept = tot;

  if (topp_on) {
    const double P = __dmul_rn((double)top_p, (double)tot);
    const u64 plim = top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
    __syncwarp();
    u64 above, w;
    const int b1 = max(warp_crossing_halves(hlo, hhi, plim, lane, above, w), 0);  // plim < total
    // level 2 (only when bin b1 lists too many): 256 sub-bins of its distance range
    const float dlo = (float)b1 * (1.0f / 16.0f);
    const float dw = b1 < WNB - 1 ? (1.0f / 16.0f) : 24.0f - dlo;  // the overflow bin: q = 0 beyond 21.5
    const float sub_scale = (float)WNB / dw;
    auto bin2 = [&](float x) -> int {
      const float z = __fmul_rn(__fsub_rn(__fsub_rn(gmax, x), dlo), sub_scale);
      return __float2int_rz(fminf(fmaxf(z, 0.0f), (float)(WNB - 1)));
    };
    int level = 1, b2 = -1;
    int m = 0;
#pragma unroll 1
    while (true) {
      // list the candidates of the crossing bin (of sub-bin b2 at level 2)
      m = 0;
#pragma unroll 1
      for (int s = 0; s < NS; ++s) {
        const int c = s * 32 + lane;
        float v[8];
        uint32_t memb = 0;
        if (c < nch) {
          load8(c, v);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            memb |= (uint32_t)(finite_val(v[e]) && v[e] >= tk && 8 * c + e < V && bin1(v[e]) == b1 &&
                               (level == 1 || bin2(v[e]) == b2)) << e;
        }
        const uint32_t cnt = __popc(memb);
        const uint32_t incl = warp_incl_scan_u32(cnt, lane);
        int pos = m + (int)(incl - cnt);
        if (memb) {
          uint32_t q[8];
          mass8(c, v, q);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if ((memb >> e) & 1u) {
              if (pos < WMINI) {
                mx[pos] = v[e];
                mi[pos] = 8 * c + e;
                mq[pos] = q[e];
              }
              ++pos;
            }
        }
        m += (int)__shfl_sync(FULL, incl, 31);
      }
      __syncwarp();
      if (m <= WMINI) break;
      if (level == 2) {
        out->ok = 0;  // the radix path takes the row
        return;
      }
      // split bin b1 into 256 sub-bins of its distance range
      zero_hist();
#pragma unroll 1
      for (int s = 0; s < NS; ++s) {
        const int c = s * 32 + lane;
        if (c >= nch) break;
        float v[8];
        load8(c, v);
        uint32_t memb = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          memb |= (uint32_t)(finite_val(v[e]) && v[e] >= tk && 8 * c + e < V && bin1(v[e]) == b1) << e;
        if (memb) {
          uint32_t q[8];
          mass8(c, v, q);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (((memb >> e) & 1u) && q[e]) {
              const int b = bin2(v[e]);
              atomicAdd(hlo + b, q[e] & 0xffffu);
              atomicAdd(hhi + b, q[e] >> 16);
            }
        }
      }
      __syncwarp();
      u64 above2, w2;
      b2 = max(warp_crossing_halves(hlo, hhi, plim - above, lane, above2, w2), 0);  // plim - above < w
      above += above2;
      level = 2;
    }
    // canonical order inside the final bin: the candidate whose mass prefix crosses plim
    float my_x = 0.0f;
    int32_t my_id = NO_ID;
    u64 my_q = 0;
    bool found = false;
#pragma unroll 1
    for (int j = lane; j < m; j += 32) {
      const float xj = mx[j];
      const int32_t ij = mi[j];
      u64 am = above;
#pragma unroll 1
      for (int jj = 0; jj < m; ++jj)
        if (canon_before(mx[jj], mi[jj], xj, ij)) am += mq[jj];
      if (mq[j] != 0u && am <= plim && am + mq[j] > plim) {
        my_x = xj;
        my_id = ij;
        my_q = am + mq[j];
        found = true;
      }
    }
    const unsigned bf = __ballot_sync(FULL, found);
    const int src = max(__ffs(bf) - 1, 0);
    out->cut_x = __shfl_sync(FULL, my_x, src);
    out->cut_id = __shfl_sync(FULL, my_id, src);
    qkept = __shfl_sync(FULL, my_q, src);
    out->topp_cut = 1;
    bool tie = false;
#pragma unroll 1
    for (int j = lane; j < m; j += 32) tie |= mx[j] == out->cut_x && mi[j] > out->cut_id;
    if (__any_sync(FULL, tie)) out->status |= MTR_ROW_TIE_AT_CUT;
    __syncwarp();
  }
  out->qkept = qkept;

  // ---- the draw: id slots in order, one warp scan of the kept masses per slot
  if (sample) {
    const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
    const bool cut = out->topp_cut != 0;
    const float cx = out->cut_x;
    const int32_t cid = out->cut_id;
    u64 run = 0;
    int32_t tok = NO_ID;
#pragma unroll 1
    for (int s = 0; s < NS; ++s) {
      const int c = s * 32 + lane;
      uint32_t q[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      u64 cs = 0;
      if (c < nch) {
        float v[8];
        load8(c, v);
        mass8(c, v, q);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (cut && !(v[e] > cx || (v[e] == cx && 8 * c + e <= cid))) q[e] = 0u;
          cs += q[e];
        }
      }
      const u64 incl = warp_incl_scan_u64(cs, lane);
      const u64 tsum = __shfl_sync(FULL, incl, 31);
      if (run + tsum > R) {
        const u64 lo = run + incl - cs;
        if (cs != 0 && lo <= R && R < lo + cs) {
          u64 acc = lo;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            acc += q[e];
            if (tok == NO_ID && acc > R) tok = 8 * c + e;
          }
        }
        break;
      }
      run += tsum;
    }
    out->token = __reduce_min_sync(FULL, tok);
  }
}

template <typename Tin, bool CFG>
__global__ void __launch_bounds__(32, 10) row_warp_kernel(const __grid_constant__ MtrSamplerArgs a,
                                                         const __grid_constant__ Derived dv) {
  wait_prior_grid();
  using E = Elem<Tin>;
  constexpr int VEC = E::VEC;            // elements per 16-byte group
  constexpr int NV = 8 / VEC;            // 16-byte groups per 8-id chunk and side
  constexpr bool SPLIT = sizeof(Tin) == 2;
  constexpr int NS = WV_MAX / 256;       // chunk slots per lane
  __shared__ __align__(8) uint64_t mbar;
  extern __shared__ __align__(16) uint8_t dsm[];
  const int lane = threadIdx.x;
  const int V = a.vocab;
  const int VP = warp_vpad(V);
  const int HALF = VP / 2;
  const int nch = (V + 7) / 8;
  float* X = (float*)dsm;
  uint8_t* U = dsm + (size_t)VP * 4;
  uint32_t* cnt = (uint32_t*)U;          // chain: u8 history counts, four per word (exact path: u16, two per word)
  u64* hist = (u64*)U;                   // selection
  uint32_t* hc = (uint32_t*)U;
  float* lx = (float*)(U + WNB * 8);
  int32_t* lid = (int32_t*)(lx + WCAP);
  uint32_t* lq = (uint32_t*)(lid + WCAP);
  float* mx = (float*)(lq + WCAP);
  int32_t* mi = (int32_t*)(mx + WMINI);
  uint32_t* mq = (uint32_t*)(mi + WMINI);
  const int L = a.input_ids ? dv.ids_len : 0;
  const float NEG = neg_inf();
  const int sel = a.select_mode;
  const bool force_radix = (a.flags & MTR_FLAG_FORCE_RADIX) != 0;
  const bool bulk = dv.vec_ok != 0;
  const uint32_t row_bytes = (uint32_t)V * (uint32_t)sizeof(Tin);
  const u64 NEG1 = pk2(dv.neg_one, dv.neg_one), NZ = pk2(dv.neg_zero, dv.neg_zero), ONE = pk2(dv.one, dv.one);
  const u64 SC = pk2(a.cfg_scale, a.cfg_scale);
  const bool pen_temp = dv.pen_on && (a.temp_mode == MTR_TEMP_COLUMN_RANGES || a.temp_mode == MTR_TEMP_ROW_CONDITIONAL ||
                                      a.temperature != 1.0f);

  auto lo_of = [&](int c) -> float* { return X + (SPLIT ? 4 * c : 8 * c); };
  auto hi_of = [&](int c) -> float* { return X + (SPLIT ? HALF + 4 * c : 8 * c + 4); };
  auto xat = [&](int id) -> float* { return ((id & 4) ? hi_of(id >> 3) : lo_of(id >> 3)) + (id & 3); };
  auto issue_copy = [&](int64_t r) {  // lane 0; every lane fenced, then __syncwarp
    const Tin* s1 = (const Tin*)a.logits + r * a.logits_row_stride;
    mbar_expect_tx(&mbar, (SPLIT && CFG) ? 2u * row_bytes : row_bytes);
    bulk_g2s(X, s1, row_bytes, &mbar);
    if constexpr (SPLIT && CFG) bulk_g2s(X + HALF, s1 + dv.second * a.logits_row_stride, row_bytes, &mbar);
  };

  if (lane == 0) mbar_init(&mbar);
  __syncwarp();
  int64_t row = blockIdx.x;
  uint32_t parity = 0;
  // the first row's history ids and per-row values go out before its logits:
  // the counts and masks need them first and can then run while the logits land
  WarpAhead ah;
  if (row < a.num_rows) load_ahead(a, dv, row, lane, L, ah);
  if (bulk && lane == 0 && row < a.num_rows) issue_copy(row);
  if (row < a.num_rows) load_ahead_class(a, lane, V, L, ah);

#pragma unroll 1
  for (; row < a.num_rows; row += gridDim.x) {
    const int64_t nrow = row + gridDim.x;
    bool issued = false;
    auto issue_next = [&]() {  // the next row's copy (its per-row values follow at the call site)
      issued = true;
      fence_proxy_async();
      __syncwarp();
      if (bulk && lane == 0 && nrow < a.num_rows) issue_copy(nrow);
    };
    const Tin* r1 = (const Tin*)a.logits + row * a.logits_row_stride;
    const Tin* r2 = r1 + dv.second * a.logits_row_stride;

    // ---------------------------------------------------------- row scalars (dependent loads from the ahead values)
    uint32_t status = 0;
    int32_t mono = -1;
    uint32_t allow = 0xffffffffu;
    int gon = 0;
    const uint32_t* gbits = nullptr;
    float t_row = a.temperature, y_row = dv.temp_rcp, u = 0.0f;
    {
      int32_t m0 = -1;
      uint32_t al = 0xffffffffu, st = 0;
      int g = 0;
      u64 gb = 0;
      float t = a.temperature, y = dv.temp_rcp, uu = 0.0f;
      if (lane == 0 && a.mono_mode == MTR_MONO_STATE) {
        m0 = ah.mono;
        if ((a.flags & MTR_FLAG_MONO_UPDATE_FROM_IDS) && L > 0) m0 = mono_update(a, m0, ahead_last(a, ah, L));
      } else if (lane == 1 && a.grammar_class_of) {
        const int64_t prev = ahead_prev(a, ah, L);
        if (prev >= V) st |= MTR_ROW_BAD_ID;
        if (prev >= 0 && prev < V) {
          const uint32_t c = ah.cls;
          if (c < (uint32_t)a.grammar_n_classes) {
            g = 1;
            if (a.grammar_vocab_bits) gb = (u64)(a.grammar_vocab_bits + (size_t)c * dv.gwords);
            else al = __ldg(a.grammar_allow + c);  // the class-byte path needs the allow row
          } else {
            st |= MTR_ROW_BAD_ID;
          }
        }
      } else if (lane == 2 && a.temp_mode == MTR_TEMP_ROW_CONDITIONAL) {
        bool hit = false;  // first matching condition wins (static indices keep ah in registers)
#pragma unroll
        for (int c = 0; c < MTR_MAX_COND_TEMPS; ++c) {
          const int off = a.cond_offset[c];
          const bool have = c < a.n_cond && off >= 1 && L >= off;
          const int64_t tok = !have ? -1 : (a.ids_dtype == MTR_IDS_I32 ? (int64_t)(int32_t)ah.cond32[c] : (int64_t)ah.cond64[c]);
          if (!hit && have && tok >= 0 && tok < V &&
              ((__ldg(a.cond_token_bits[c] + (tok >> 5)) >> (tok & 31)) & 1u)) {
            t = a.cond_temperature[c];
            y = dv.cond_rcp[c];
            hit = true;
          }
        }
      } else if (lane == 3 && sel == MTR_SELECT_SAMPLE) {
        uu = __uint_as_float(ah.ubits);
        if (!(uu >= 0.0f)) {
          uu = 0.0f;
          st |= MTR_ROW_BAD_UNIFORM;
        } else if (uu >= 1.0f) {
          uu = 0x1.fffffep-1f;
          st |= MTR_ROW_BAD_UNIFORM;
        }
      }
      if (a.mono_mode == MTR_MONO_STATE) mono = __shfl_sync(FULL, m0, 0);
      allow = __shfl_sync(FULL, al, 1);
      gon = __shfl_sync(FULL, g, 1);
      gbits = (const uint32_t*)__shfl_sync(FULL, gb, 1);
      t_row = __shfl_sync(FULL, t, 2);
      y_row = __shfl_sync(FULL, y, 2);
      u = __shfl_sync(FULL, uu, 3);
      status = __reduce_or_sync(FULL, st);
    }
    if (a.mono_mode == MTR_MONO_SCAN) {
      // last time-shift position and last start-of-sequence position
      int lts = -1, lsos = -1;
      int32_t lts_id = 0;
#pragma unroll
      for (int k = 0; k < WHIST; ++k) {
        const int pos = ah.hbase + lane + 32 * k;
        const int32_t t = narrow_raw(a, ah.hid[k]);
        if (pos < L && t != INT32_MIN) {
          if (t >= a.ts_start && t < a.ts_end) {
            lts = pos;
            lts_id = t;
          }
          if (is_sos(a, t)) lsos = pos;
        }
      }
#pragma unroll 1
      for (int base = ah.hbase - 32; base > -32 && __all_sync(FULL, lts < 0 && lsos < 0); base -= 32) {
        // neither seen in the register window: walk back (long histories only)
        const int pos = base + lane;
        if (pos >= 0) {
          const int64_t t = load_id(a, row, pos);
          if (t >= a.ts_start && t < a.ts_end) {
            lts = pos;
            lts_id = (int32_t)t;
          }
          if (is_sos(a, t)) lsos = pos;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const int op = __shfl_xor_sync(FULL, lts, o);
        const int32_t oid = __shfl_xor_sync(FULL, lts_id, o);
        if (op > lts) {
          lts = op;
          lts_id = oid;
        }
        lsos = max(lsos, __shfl_xor_sync(FULL, lsos, o));
      }
      mono = (lts != -1 && lts > lsos) ? lts_id - a.ts_start : -1;
    }
    const int mono_hi = mono >= 0 ? (int32_t)min((int64_t)a.ts_end, (int64_t)a.ts_start + mono) : -1;
    const bool masks = mono_hi > a.ts_start || gon || (V & 7) != 0;
    // grammar bitmap words of this lane's 16 chunks: issued now, used after the counts
    uint32_t gw[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const int id0 = (s * 32 + lane) * 8;
      gw[s] = 0xffffffffu;
      if (gon && gbits && id0 < V) gw[s] = __ldg(gbits + (id0 >> 5));
    }

    // ---------------------------------------------------------- history counts
    uint32_t own = 0;  // bit k: this lane counted window id k first and applies its penalties
    // ids outside the register window, or an 8-bit count that wrapped: the exact
    // 16-bit counts of the penalty step
    bool exact_counts = a.penalty_start < ah.hbase;
    int32_t ht[WHIST];  // window ids inside the penalty window and [0, V), else -1
    if (dv.pen_on) {
#pragma unroll
      for (int i = 0; i < WV_MAX / 512; ++i) {
        const int w = (i * 32 + lane) * 4;
        if (w < VP / 4) *(uint4*)(cnt + w) = make_uint4(0u, 0u, 0u, 0u);
      }
      uint32_t bad = 0;
#pragma unroll
      for (int k = 0; k < WHIST; ++k) {
        const int pos = ah.hbase + lane + 32 * k;
        const bool in_window = pos >= a.penalty_start && pos < L;
        // int32 ids are held zero-extended and RAW_NONE lies above every id,
        // so one unsigned compare checks 0 <= id < V for both id types
        const bool ok = in_window && ah.hid[k] < (u64)V;
        bad |= (uint32_t)(in_window && !ok);
        ht[k] = ok ? (int32_t)ah.hid[k] : -1;
      }
      __syncwarp();
      uint32_t wrapped = 0;
#pragma unroll
      for (int h0 = 0; h0 < WHIST; h0 += WHIST / 2) {
        uint32_t old[WHIST / 2];  // a half window of atomics in flight before any result is used
#pragma unroll
        for (int k = 0; k < WHIST / 2; ++k) {
          old[k] = 0xffffffffu;
          if (ht[h0 + k] >= 0) old[k] = atomicAdd(cnt + (ht[h0 + k] >> 2), 1u << (8 * (ht[h0 + k] & 3)));
        }
#pragma unroll
        for (int k = 0; k < WHIST / 2; ++k) {
          const uint32_t c = (old[k] >> (8 * (ht[h0 + k] & 3))) & 0xffu;
          own |= (uint32_t)(ht[h0 + k] >= 0 && c == 0u) << (h0 + k);
          wrapped |= (uint32_t)(ht[h0 + k] >= 0 && c == 0xffu);  // the add carried into the next id's count
        }
      }
#pragma unroll 1
      for (int pos = a.penalty_start + lane; pos < ah.hbase; pos += 32) {  // long histories: counted exactly later
        const int64_t t = load_id(a, row, pos);
        if (t < 0 || t >= V) bad = 1;
      }
      if (__any_sync(FULL, bad)) status |= MTR_ROW_BAD_ID;
      if (__any_sync(FULL, wrapped)) exact_counts = true;
      __syncwarp();
    }

    // keep bits of this lane's 16 chunks: slot s in bits 8s .. 8s+7 of km[s >> 3]
    u64 km[2] = {~0ull, ~0ull};
    if (masks) {
      if (gon && gbits) {
        // byte (lane & 3) of each slot's bitmap word, four slots per byte permute
        const uint32_t b = (uint32_t)lane & 3u;
        const uint32_t sel = b | ((b + 4u) << 4);
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          w[q] = __byte_perm(__byte_perm(gw[4 * q], gw[4 * q + 1], sel), __byte_perm(gw[4 * q + 2], gw[4 * q + 3], sel),
                             0x5410);
        km[0] = (u64)w[0] | ((u64)w[1] << 32);
        km[1] = (u64)w[2] | ((u64)w[3] << 32);
      } else if (gon) {
        const uint32_t ncls = (uint32_t)a.grammar_n_classes;
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const int id0 = (s * 32 + lane) * 8;
          uint32_t g = 0;
#pragma unroll 1
          for (int e = 0; e < 8; ++e) {
            if (id0 + e < V) {
              const uint32_t cl = __ldg(a.grammar_class_of + id0 + e);
              g |= (cl < ncls ? (allow >> cl) & 1u : 0u) << e;
            }
          }
          km[s >> 3] &= ~((u64)(~g & 0xffu) << (8 * (s & 7)));
        }
      }
      // clear the bits of ids [lo, hi) in this lane's slots
      auto clear_ids = [&](int lo, int hi) {
        // whole chunks: slot s (ids 256 s + 8 lane ..) inside [lo, hi)
        const int A = lo - 8 * lane, B = hi - 8 * lane - 8;
        const int s_a = A <= 0 ? 0 : (A + 255) >> 8;
        const int s_b = B < 0 ? -1 : min(B >> 8, NS - 1);
        if (s_b >= s_a) {
          const int b0 = 8 * s_a, b1 = 8 * (s_b + 1);  // bit range over the 128-bit mask
          auto bits64 = [](int l, int h) -> u64 {
            l = max(l, 0);
            h = min(h, 64);
            if (h <= l) return 0ull;
            return (h >= 64 ? ~0ull : ((1ull << h) - 1ull)) & ~((1ull << l) - 1ull);
          };
          km[0] &= ~bits64(b0, b1);
          km[1] &= ~bits64(b0 - 64, b1 - 64);
        }
        // partial chunks at either end belong to one lane each
#pragma unroll
        for (int end = 0; end < 2; ++end) {
          const int x = end == 0 ? lo : hi - 1;
          const int c = x >> 3;
          if ((c & 31) == lane && (c >> 5) < NS) {
            const int sl = c >> 5;
            const uint32_t rb = range_bits(lo - 8 * c, hi - 8 * c);
            km[sl >> 3] &= ~((u64)rb << (8 * (sl & 7)));
          }
        }
      };
      if (mono_hi > a.ts_start) clear_ids(a.ts_start, mono_hi);
      if (V & 7) clear_ids(V, nch * 8);  // the ragged tail of the last chunk
    }

    // ---------------------------------------------------------- this row's logits
    bool lost = false;
    if (bulk) {
      // the test hook gives the first wait no polls at all (the copy is still in flight)
      const bool hook = (a.flags & MTR_FLAG_TEST_COPY_TIMEOUT) && row == (int64_t)blockIdx.x;
      lost = !mbar_wait(&mbar, parity, hook ? 0u : WAIT_POLLS);
      parity ^= 1u;
      if (__any_sync(FULL, lost)) {
        // this row and every later row of this CTA are not processed: each gets
        // pad_id and MTR_ROW_COPY_TIMEOUT, so no row keeps a previous step's token
#pragma unroll 1
        for (int64_t r = row + (int64_t)lane * gridDim.x; r < a.num_rows; r += (int64_t)32 * gridDim.x) {
          if (a.out_status) a.out_status[r] = (r == row ? status : 0u) | MTR_ROW_COPY_TIMEOUT;
          if (sel != MTR_SELECT_NONE && a.out_ids) a.out_ids[r] = a.pad_id;
          if (sel != MTR_SELECT_NONE && a.id_buffer) {
            const int32_t cur = a.cur_len_dev ? *a.cur_len_dev : a.cur_len;
            if (cur >= 0 && (int64_t)cur < a.id_buffer_row_stride) a.id_buffer[r * a.id_buffer_row_stride + cur] = a.pad_id;
          }
        }
        mbar_wait(&mbar, parity ^ 1u);  // bounded: a late copy still owns X
        return;
      }
    }

    // ---------------------------------------------------------- pass 1 (in place): CFG, bias, [temperature], masks
    // Masks only ever write -inf, which bias, penalties and temperature map to
    // -inf again, so the order here (masks before or after temperature)
    // reproduces CFG -> masks -> bias -> penalties -> temperature exactly.
    // The common case (16-bit rows staged in place, no bias, no temperature in
    // this pass) runs a loop with every launch-uniform test hoisted out of it.
    bool fast_pass = false;
    if constexpr (SPLIT) {
      fast_pass = bulk && a.timeshift_bias == 0.0f &&
                  (dv.pen_on || (a.temp_mode == MTR_TEMP_SCALAR && t_row == 1.0f));
    }
    if (fast_pass) {
      if constexpr (SPLIT) {
        float* const Xlo = X + 4 * lane;
        float* const Xhi = X + HALF + 4 * lane;
        u64 kcur = km[0];  // keep bits of slot s in the low byte
#pragma unroll 4
        for (int s = 0; s < NS; ++s) {
          if ((s * 32 + lane) * 8 >= V) break;
          const uint4 ra = *(const uint4*)(Xlo + 128 * s);
          float v[8];
          if constexpr (CFG) {
            const uint4 rb = *(const uint4*)(Xhi + 128 * s);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const u64 A = pk2(E::get(ra, e), E::get(ra, e + 1));
              const u64 B = pk2(E::get(rb, e), E::get(rb, e + 1));
              up2(fma2(fma2(fma2(B, NEG1, A), SC, NZ), ONE, B), v[e], v[e + 1]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = E::get(ra, e);
          }
          if (masks) {
            const uint32_t keep = (uint32_t)kcur;
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = ((keep >> e) & 1u) ? v[e] : NEG;
          }
          kcur = s == 7 ? km[1] : kcur >> 8;
          *(float4*)(Xlo + 128 * s) = make_float4(v[0], v[1], v[2], v[3]);
          *(float4*)(Xhi + 128 * s) = make_float4(v[4], v[5], v[6], v[7]);
        }
      }
    } else {
#pragma unroll 1
      for (int s = 0; s < NS; ++s) {
        const int c = s * 32 + lane;
        const int id0 = c * 8;
        if (id0 >= V) continue;
        uint4 ra[NV];
#pragma unroll
        for (int h = 0; h < NV; ++h) {
          if (bulk) ra[h] = *(const uint4*)(lo_of(c) + 4 * h);
          else ra[h] = E::gather(r1, id0 + h * VEC, V);
        }
        float v[8];
        if constexpr (CFG) {
          uint4 rb[NV];
#pragma unroll
          for (int h = 0; h < NV; ++h) {
            if (SPLIT && bulk) rb[h] = *(const uint4*)(hi_of(c) + 4 * h);
            else if (bulk) rb[h] = __ldcs((const uint4*)(r2 + id0 + h * VEC));
            else rb[h] = E::gather(r2, id0 + h * VEC, V);
          }
          // b + (a - b) * s as three FMAs whose -1 / -0 / 1 operands are launch
          // parameters, so the compiler cannot form a fusable mul + add pair
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const u64 A = pk2(E::get(ra[e / VEC], e % VEC), E::get(ra[e / VEC], e % VEC + 1));
            const u64 B = pk2(E::get(rb[e / VEC], e % VEC), E::get(rb[e / VEC], e % VEC + 1));
            up2(fma2(fma2(fma2(B, NEG1, A), SC, NZ), ONE, B), v[e], v[e + 1]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = E::get(ra[e / VEC], e % VEC);
        }
        if (a.timeshift_bias != 0.0f) {
          const uint32_t bb = range_bits(a.ts_start - id0, a.ts_end - id0);
          if (bb) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if ((bb >> e) & 1u) v[e] = __fadd_rn(v[e], a.timeshift_bias);
          }
        }
        if (!dv.pen_on) temp_chunk(a, dv, v, id0, t_row, y_row);
        if (masks) {
          const uint32_t keep = (uint32_t)((s < 8 ? km[0] : km[1]) >> (8 * (s & 7)));
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = ((keep >> e) & 1u) ? v[e] : NEG;
        }
        *(float4*)lo_of(c) = make_float4(v[0], v[1], v[2], v[3]);
        *(float4*)hi_of(c) = make_float4(v[4], v[5], v[6], v[7]);
      }
    }

    // ---------------------------------------------------------- penalties: one lane per distinct history id
    if (dv.pen_on) {
      __syncwarp();
      const float rp = a.repetition_penalty, fp = a.frequency_penalty, pp = a.presence_penalty;
      // repetition (x < 0 ? x * rp : x / rp), then frequency and presence; with
      // rp = 1, fp = 0 or pp = 0 the step is the identity, so the common loop
      // skips none (pen_value, used out of line, skips them)
      if (!exact_counts) {
        // the lane that counted an id first applies it, with the final count;
        // per half of the window: loads first, then the arithmetic, then the stores
        const float y = dv.rep_rcp;
#pragma unroll
        for (int h0 = 0; h0 < WHIST; h0 += WHIST / 2) {
          float xv[WHIST / 2];
          uint32_t cw[WHIST / 2];
          int xo[WHIST / 2];
#pragma unroll
          for (int k = 0; k < WHIST / 2; ++k) {
            const int32_t t = ((own >> (h0 + k)) & 1u) ? ht[h0 + k] : 0;
            xo[k] = SPLIT ? ((t & 4) ? HALF : 0) + ((t >> 3) << 2) + (t & 3) : t;  // float index of id t in X
            xv[k] = X[xo[k]];
            cw[k] = cnt[t >> 2];
          }
          bool rare = false;
#pragma unroll
          for (int k = 0; k < WHIST / 2; ++k) {
            const int32_t t = ((own >> (h0 + k)) & 1u) ? ht[h0 + k] : 0;
            const float c = (float)((cw[k] >> (8 * (t & 3))) & 0xffu);
            const float x = xv[k];
            const float ax = fabsf(x);
            // x / rp by Markstein for normal-range positive x; other operands go out of line
            const float q0 = __fmul_rn(x, y);
            const float q = __fmaf_rn(__fmaf_rn(-q0, rp, x), y, q0);
            rare |= ((own >> (h0 + k)) & 1u) && !(x < 0.0f) && !(y != 0.0f && ax >= 0x1p-60f && ax < 0x1p60f);
            float r = x < 0.0f ? __fmul_rn(x, rp) : q;
            r = __fsub_rn(r, __fmul_rn(fp, c));
            xv[k] = __fsub_rn(r, pp);
          }
          if (__any_sync(FULL, rare)) {
            PenIds8 ids;
#pragma unroll
            for (int k = 0; k < WHIST / 2; ++k) ids.t[k] = ((own >> (h0 + k)) & 1u) ? ht[h0 + k] : 0;
            pen_rare8(X, cnt, ids, (own >> h0) & 0xffu, HALF, SPLIT, rp, fp, pp, dv.rep_rcp);
          } else {
#pragma unroll
            for (int k = 0; k < WHIST / 2; ++k)
              if ((own >> (h0 + k)) & 1u) X[xo[k]] = xv[k];
          }
        }
      } else {
        pen_exact(X, cnt, a, row, L, V, VP, SPLIT, lane, rp, fp, pp, dv.rep_rcp);
      }
      __syncwarp();
      if (pen_temp) {
#pragma unroll 1
        for (int s = 0; s < NS; ++s) {
          const int c = s * 32 + lane;
          const int id0 = c * 8;
          if (id0 >= V) break;
          const float4 f0 = *(const float4*)lo_of(c), f1 = *(const float4*)hi_of(c);
          float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
          temp_chunk(a, dv, v, id0, t_row, y_row);
          *(float4*)lo_of(c) = make_float4(v[0], v[1], v[2], v[3]);
          *(float4*)hi_of(c) = make_float4(v[4], v[5], v[6], v[7]);
        }
      }
    }
    __syncwarp();

    // ---------------------------------------------------------- chunk maxima (NaN propagates)
    float cm[NS];
    float lmax = NEG;
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      const int c = s * 32 + lane;
      cm[s] = NEG;
      if (c < nch) {
        const float4 f0 = *(const float4*)lo_of(c), f1 = *(const float4*)hi_of(c);
        cm[s] = fmax3n(fmax3n(f0.x, f0.y, f0.z), fmax3n(f0.w, f1.x, f1.y), fmax2n(f1.z, f1.w));
        lmax = fmax2n(lmax, cm[s]);
      }
    }
    float gmax = lmax;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gmax = fmax2n(gmax, __shfl_xor_sync(FULL, gmax, o));
    const bool has_nan = gmax != gmax;
    const bool nonfinite = has_nan || gmax == pos_inf();
    const bool all_masked = !nonfinite && gmax == NEG;
    if (nonfinite) status |= MTR_ROW_NONFINITE;
    if (all_masked) status |= MTR_ROW_ALL_MASKED;
    const bool clean = !nonfinite && !all_masked;
    const bool want_lp = a.out_logprobs != nullptr;
    const bool need_x_late = a.out_scores != nullptr || want_lp;
    const bool need_mass = clean && (sel == MTR_SELECT_SAMPLE || want_lp || (sel == MTR_SELECT_NONE && dv.topp_on));

    float tk = NEG;
    bool topp_cut = false;
    float cut_x = 0.0f;
    int32_t cut_id = NO_ID;
    u64 qkept = 0;
    int32_t token = -1;
    int n = -1;  // survivors listed in lx / lid (-1: no list)
    bool small = false;  // mx / mi hold the candidates (<= 64), not yet cut to the top k
    bool small128 = false;  // lx / lid hold 65 .. 128 candidates, not yet cut to the top k

    if (sel == MTR_SELECT_ARGMAX && !all_masked) {
      // lowest id of the maximum (of the first NaN when there is one)
      int32_t myc = NO_ID;
#pragma unroll
      for (int s = NS - 1; s >= 0; --s)
        if (has_nan ? cm[s] != cm[s] : cm[s] == gmax) myc = s * 32 + lane;
      myc = __reduce_min_sync(FULL, myc);
      int32_t hit = NO_ID;
      if (myc < nch && lane < 8) {
        const int id = myc * 8 + lane;
        const float v = *xat(id);
        if (has_nan ? v != v : v == gmax) hit = id;
      }
      token = __reduce_min_sync(FULL, hit);
      if (token == NO_ID) token = 0;
    } else if (sel == MTR_SELECT_ARGMAX) {
      token = 0;
    } else if (clean && dv.topk_on) {
      const uint32_t k = (uint32_t)a.top_k;
      bool topk_done = false;
      if (!force_radix) {
        // bound: the chunk maxima in bins <= btau number >= k, so >= k scores lie
        // within chi of the max.  btau from a shared histogram of the 64 nearest
        // bins; beyond them, a binary search over the 256 bins whose probes count
        // this lane's slots at or below the probe and sum over the warp.
        uint32_t wbp[NS / 4];  // the slots' bins, four per word (255: empty slot)
#pragma unroll
        for (int q = 0; q < NS / 4; ++q) {
          uint32_t w = 0;
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float x = cm[4 * q + r];
            w |= (uint32_t)(x > NEG ? wbin(gmax, x) : WNB - 1) << (8 * r);
          }
          wbp[q] = w;
        }
        auto count_le = [&](int b) -> uint32_t {  // chunk maxima in bins <= b (b < 255)
          uint32_t c = 0;
#pragma unroll
          for (int q = 0; q < NS / 4; ++q)
#pragma unroll
            for (int r = 0; r < 4; ++r) c += ((wbp[q] >> (8 * r)) & 0xffu) <= (uint32_t)b;
          return __reduce_add_sync(FULL, c);
        };
        int btau = WNB - 1;  // overflow: no bound
        {
          // the bound usually lies within 8 logits of the max: a 64-bin shared histogram
          // of those bins (two per lane) and one scan find it
          *(uint2*)(hc + 2 * lane) = make_uint2(0u, 0u);
          __syncwarp();
#pragma unroll
          for (int q = 0; q < NS / 4; ++q)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const uint32_t bq = (wbp[q] >> (8 * r)) & 0xffu;
              if (bq < 64u) atomicAdd(hc + bq, 1u);
            }
          __syncwarp();
          const uint2 hp = *(const uint2*)(hc + 2 * lane);
          const uint32_t incl = warp_incl_scan_u32(hp.x + hp.y, lane);
          const unsigned bal = __ballot_sync(FULL, incl >= k);
          if (bal) {
            const int l = __ffs(bal) - 1;  // first lane whose bins reach k
            const uint32_t before = __shfl_sync(FULL, incl - hp.x - hp.y, l);
            const uint32_t h0 = __shfl_sync(FULL, hp.x, l);
            btau = 2 * l + (before + h0 >= k ? 0 : 1);
          } else if (count_le(WNB - 2) >= k) {
            int lo = 64, hi = WNB - 2;  // smallest b with count_le(b) >= k lies in [lo, hi]
#pragma unroll 1
            while (lo < hi) {
              const int mid = (lo + hi) >> 1;
              if (count_le(mid) >= k) hi = mid;
              else lo = mid + 1;
            }
            btau = lo;
          }
          __syncwarp();
        }
        if (btau < WNB - 1) {  // the overflow bin bounds nothing
          const float chi = (float)(btau + 1) * (1.0f / WBIN_SCALE);
          uint32_t qual = 0;
#pragma unroll
          for (int q = 0; q < NS / 4; ++q)
#pragma unroll
            for (int r = 0; r < 4; ++r) qual |= (uint32_t)(((wbp[q] >> (8 * r)) & 0xffu) <= (uint32_t)btau) << (4 * q + r);
          // each lane lists the scores of its qualifying chunks within chi of the max:
          // count (keeping each chunk's 8-bit hit mask), one warp scan for the offsets,
          // then store at the final positions -- no shared counter, no overflow
          int cl = 0;
          u64 hm[2] = {0ull, 0ull};  // hit mask of slot s in byte s & 7 of hm[s >> 3]
          {
            uint32_t qq = qual;
#pragma unroll 1
            while (qq) {
              const int s = __ffs(qq) - 1;
              qq &= qq - 1u;
              const int c = s * 32 + lane;
              const float4 f0 = *(const float4*)lo_of(c), f1 = *(const float4*)hi_of(c);
              const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
              uint32_t cmask = 0;
#pragma unroll
              for (int e = 0; e < 8; ++e) cmask |= (uint32_t)(__fsub_rn(gmax, v[e]) < chi) << e;
              cl += __popc(cmask);
              if (s < 8) hm[0] |= (u64)cmask << (8 * s);
              else hm[1] |= (u64)cmask << (8 * (s - 8));
            }
          }
          const uint32_t incl = warp_incl_scan_u32((uint32_t)cl, lane);
          const int total = (int)__shfl_sync(FULL, incl, 31);
          if (total <= WCAP) {
            // small lists go straight to the sort's arrays
            float* dx = total <= 64 ? mx : lx;
            int32_t* di = total <= 64 ? mi : lid;
            int pos = (int)incl - cl;
            uint32_t qq = qual;
#pragma unroll 1
            while (qq) {
              const int s = __ffs(qq) - 1;
              qq &= qq - 1u;
              const uint32_t cmask = (uint32_t)((s < 8 ? hm[0] : hm[1]) >> (8 * (s & 7))) & 0xffu;
              if (cmask == 0u) continue;
              const int c = s * 32 + lane;
              const float4 f0 = *(const float4*)lo_of(c), f1 = *(const float4*)hi_of(c);
              const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
              for (int e = 0; e < 8; ++e)
                if ((cmask >> e) & 1u) {
                  const int p = pos + __popc(cmask & ((1u << e) - 1u));
                  dx[p] = v[e];
                  di[p] = c * 8 + e;
                }
              pos += __popc(cmask);
            }
          }
          __syncwarp();
          if (total <= 64) {
            n = total;
            small = true;
            topk_done = true;
          } else if (total <= 128) {
            n = total;
            small128 = true;
            topk_done = true;
          } else if (total <= WCAP) {
            n = total;
            // exact k-th value: fine histogram over the list, then the crossing bin
            const float s2 = (float)WNB / chi;
            auto fbin = [&](float x) -> int {
              float z = __fmul_rn(__fsub_rn(gmax, x), s2);
              z = fminf(z, (float)(WNB - 1));
              return __float2int_rz(z);
            };
#pragma unroll 1
            for (int i = lane * 4; i < WNB; i += 128) *(uint4*)(hc + i) = make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
#pragma unroll 1
            for (int j = lane; j < n; j += 32) atomicAdd(hc + fbin(lx[j]), 1u);
            __syncwarp();
            u64 above2, w2;
            const int b2 = max(warp_crossing(hc, (u64)(k - 1), lane, above2, w2), 0);  // n >= k
            int m = 0;
#pragma unroll 1
            for (int j0 = 0; j0 < n; j0 += 32) {
              const int j = j0 + lane;
              const bool in = j < n && fbin(lx[j]) == b2;
              const unsigned bm = __ballot_sync(FULL, in);
              const int pos = m + __popc(bm & ((1u << lane) - 1u));
              if (in && pos < WMINI) mx[pos] = lx[j];
              m += __popc(bm);
            }
            __syncwarp();
            float my_tk = NEG;
            bool found = false;
            if (m <= WMINI) {
#pragma unroll 1
              for (int j = lane; j < m; j += 32) {
                const float xi = mx[j];
                uint32_t gt = 0, ge = 0;
#pragma unroll 1
                for (int jj = 0; jj < m; ++jj) {
                  gt += mx[jj] > xi;
                  ge += mx[jj] >= xi;
                }
                if (above2 + gt <= k - 1 && k - 1 < above2 + ge) {
                  my_tk = xi;
                  found = true;
                }
              }
            } else {
#pragma unroll 1
              for (int j = lane; j < n; j += 32) {
                const float xi = lx[j];
                uint32_t gt = 0, ge = 0;
#pragma unroll 1
                for (int jj = 0; jj < n; ++jj) {
                  gt += lx[jj] > xi;
                  ge += lx[jj] >= xi;
                }
                if (gt <= k - 1 && k - 1 < ge) {
                  my_tk = xi;
                  found = true;
                }
              }
            }
            const unsigned bal3 = __ballot_sync(FULL, found);
            tk = __shfl_sync(FULL, my_tk, max(__ffs(bal3) - 1, 0));
            // keep the survivors (x >= tk) at the front of the list
            float sx[WCAP / 32];
            int32_t si[WCAP / 32];
#pragma unroll
            for (int t2 = 0; t2 < WCAP / 32; ++t2) {
              const int j = lane + 32 * t2;
              sx[t2] = j < n ? lx[j] : NEG;
              si[t2] = j < n ? lid[j] : 0;
            }
            __syncwarp();
            int base = 0;
#pragma unroll
            for (int t2 = 0; t2 < WCAP / 32; ++t2) {
              const bool keepj = sx[t2] >= tk && sx[t2] > NEG;
              const unsigned bm = __ballot_sync(FULL, keepj);
              if (keepj) {
                const int pos = base + __popc(bm & ((1u << lane) - 1u));
                lx[pos] = sx[t2];
                lid[pos] = si[t2];
              }
              base += __popc(bm);
            }
            __syncwarp();
            n = base;
            topk_done = true;
          }
        }
      }
      if (!topk_done) {
        // exact k-th over the whole row: count, then radix select over X
        uint32_t nf = 0;
#pragma unroll 1
        for (int c = lane; c < nch; c += 32) {
          const float4 f0 = *(const float4*)lo_of(c), f1 = *(const float4*)hi_of(c);
          nf += finite_val(f0.x) + finite_val(f0.y) + finite_val(f0.z) + finite_val(f0.w) + finite_val(f1.x) +
                finite_val(f1.y) + finite_val(f1.z) + finite_val(f1.w);
        }
        nf = __reduce_add_sync(FULL, nf);
        n = -1;
        if (k < nf) {
          status |= MTR_ROW_SLOW_PATH;
          uint32_t prefix = 0, mask = 0;
          u64 above = 0, wlast = 0;
#pragma unroll 1
          for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll 1
            for (int i = lane * 4; i < WNB; i += 128) *(uint4*)(hc + i) = make_uint4(0u, 0u, 0u, 0u);
            __syncwarp();
#pragma unroll 1
            for (int id = lane; id < V; id += 32) {
              const float x = *xat(id);
              if (finite_val(x)) {
                const uint32_t key = fkey(x);
                if ((key & mask) == prefix) atomicAdd(hc + (255 - (int)((key >> shift) & 255u)), 1u);
              }
            }
            __syncwarp();
            u64 ab;
            const int b = max(warp_crossing(hc, (u64)(k - 1) - above, lane, ab, wlast), 0);  // k <= finite count
            above += ab;
            prefix |= (255u - (uint32_t)b) << shift;
            mask |= 255u << shift;
            __syncwarp();
          }
          tk = key2f(prefix);
          const u64 nge = above + wlast;
          if (nge <= (u64)WCAP && !force_radix) {
            // list the survivors in id order
            int base = 0;
#pragma unroll 1
            for (int id0 = 0; id0 < V; id0 += 32) {
              const int id = id0 + lane;
              float x = NEG;
              if (id < V) x = *xat(id);
              const bool keepj = finite_val(x) && x >= tk;
              const unsigned bm = __ballot_sync(FULL, keepj);
              const int pos = base + __popc(bm & ((1u << lane) - 1u));
              if (keepj && pos < WCAP) {
                lx[pos] = x;
                lid[pos] = id;
              }
              base += __popc(bm);
            }
            __syncwarp();
            n = min(base, WCAP);
          }
        }
      }
    }
    if (!need_x_late && n >= 0) {  // X is no longer read by this row
      issue_next();
      if (nrow < a.num_rows) load_ahead(a, dv, nrow, lane, L, ah);
    }

    // ---------------------------------------------------------- top-p and the draw
    if (small) {
      // at most 64 candidates: one bitonic sort in canonical order (score desc,
      // id asc) gives the k-th score, the top-p cut is a prefix scan, and a
      // second sort of the kept entries by id gives the draw
      const uint32_t k = (uint32_t)a.top_k;
      const int j0 = 2 * lane, j1 = j0 + 1;
      u64 a0 = j0 < n ? (((u64)fkey(mx[j0]) << 32) | (u64)(~(uint32_t)mi[j0])) : 0ull;
      u64 a1 = j1 < n ? (((u64)fkey(mx[j1]) << 32) | (u64)(~(uint32_t)mi[j1])) : 0ull;
      sort64_desc(a0, a1, lane);
      const int p = (int)k - 1;
      const u64 v0 = __shfl_sync(FULL, a0, p >> 1), v1 = __shfl_sync(FULL, a1, p >> 1);
      const uint32_t tkey = (uint32_t)(((p & 1) ? v1 : v0) >> 32);
      tk = key2f(tkey);
      const bool s0 = a0 != 0ull && (uint32_t)(a0 >> 32) >= tkey, s1 = a1 != 0ull && (uint32_t)(a1 >> 32) >= tkey;
      uint32_t q0 = 0, q1 = 0;
      if (need_mass) {
        expfx2(__fsub_rn(key2f((uint32_t)(a0 >> 32)), gmax), __fsub_rn(key2f((uint32_t)(a1 >> 32)), gmax), q0, q1);
        q0 = s0 ? q0 : 0u;
        q1 = s1 ? q1 : 0u;
        const u64 lsum = (u64)q0 + q1;
        const u64 incl = warp_incl_scan_u64(lsum, lane);
        qkept = __shfl_sync(FULL, incl, 31);
        int pcut = 64;
        if (dv.topp_on) {
          const double P = __dmul_rn((double)a.top_p, (double)qkept);
          const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
          const u64 ab0 = incl - lsum, ab1 = ab0 + q0;
          int my = -1;
          u64 myq = 0;
          if (q0 != 0u && ab0 <= plim && ab0 + q0 > plim) {
            my = j0;
            myq = ab0 + q0;
          } else if (q1 != 0u && ab1 <= plim && ab1 + q1 > plim) {
            my = j1;
            myq = ab1 + q1;
          }
          const unsigned bal = __ballot_sync(FULL, my >= 0);
          const int src = max(__ffs(bal) - 1, 0);
          pcut = max(__shfl_sync(FULL, my, src), 0);
          qkept = __shfl_sync(FULL, myq, src);
          const int pn = min(pcut + 1, 63);
          const u64 c0 = __shfl_sync(FULL, a0, pcut >> 1), c1 = __shfl_sync(FULL, a1, pcut >> 1);
          const u64 n0 = __shfl_sync(FULL, a0, pn >> 1), n1 = __shfl_sync(FULL, a1, pn >> 1);
          const u64 ck = (pcut & 1) ? c1 : c0, nk = (pn & 1) ? n1 : n0;
          cut_x = key2f((uint32_t)(ck >> 32));
          cut_id = (int32_t)(~(uint32_t)ck);
          topp_cut = true;
          if (pcut + 1 < 64 && nk != 0ull && (uint32_t)(nk >> 32) == (uint32_t)(ck >> 32)) status |= MTR_ROW_TIE_AT_CUT;
        }
        if (sel == MTR_SELECT_SAMPLE) {
          // the smallest id whose id-ordered kept mass exceeds R: the kept mass of
          // 32 id buckets (low and high 16 bits of q summed apart, so the shared
          // atomics are 32-bit), a warp scan for the bucket where the mass crosses
          // R, then the few kept entries inside that bucket
          const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
          const bool kp0 = q0 != 0u && j0 <= pcut, kp1 = q1 != 0u && j1 <= pcut;
          const int i0 = (int)(~(uint32_t)a0), i1 = (int)(~(uint32_t)a1);
          int bsh = 3;  // bucket width 2^bsh: 32 buckets cover [0, VP)
          while ((32 << bsh) < VP) ++bsh;
          uint32_t* const bk = hc;  // bucket b: low-half sum at bk[2b], high-half sum at bk[2b + 1]
          *(uint2*)(bk + 2 * lane) = make_uint2(0u, 0u);
          __syncwarp();
          if (kp0) {
            atomicAdd(bk + 2 * (i0 >> bsh), q0 & 0xffffu);
            atomicAdd(bk + 2 * (i0 >> bsh) + 1, q0 >> 16);
          }
          if (kp1) {
            atomicAdd(bk + 2 * (i1 >> bsh), q1 & 0xffffu);
            atomicAdd(bk + 2 * (i1 >> bsh) + 1, q1 >> 16);
          }
          __syncwarp();
          const uint2 hh = *(const uint2*)(bk + 2 * lane);
          const u64 hb = ((u64)hh.y << 16) + hh.x;
          const u64 incl = warp_incl_scan_u64(hb, lane);
          const int b = max(__ffs(__ballot_sync(FULL, incl > R)) - 1, 0);  // the total qkept exceeds R
          u64 f0 = __shfl_sync(FULL, incl - hb, b), f1 = f0;
          const bool in0 = kp0 && (i0 >> bsh) == b, in1 = kp1 && (i1 >> bsh) == b;
          unsigned m0 = __ballot_sync(FULL, in0), m1 = __ballot_sync(FULL, in1);
#pragma unroll 1
          while (m0 | m1) {  // each entry of the bucket adds its mass to the entries at or above its id
            const bool from0 = m0 != 0u;
            const int src = __ffs(from0 ? m0 : m1) - 1;
            if (from0) m0 &= m0 - 1u;
            else m1 &= m1 - 1u;
            const int is = __shfl_sync(FULL, from0 ? i0 : i1, src);
            const uint32_t qs = __shfl_sync(FULL, from0 ? q0 : q1, src);
            f0 += is <= i0 ? qs : 0u;
            f1 += is <= i1 ? qs : 0u;
          }
          int32_t my = NO_ID;
          if (in0 && f0 > R && f0 - q0 <= R) my = i0;
          if (in1 && f1 > R && f1 - q1 <= R) my = i1;
          token = __reduce_min_sync(FULL, my);
        }
      }
    } else if (small128) {
      // 65 .. 128 candidates: the same steps on one 128-key sort, four keys per lane
      const uint32_t k = (uint32_t)a.top_k;
      u64 kk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = 4 * lane + e;
        kk[e] = j < n ? (((u64)fkey(lx[j]) << 32) | (u64)(~(uint32_t)lid[j])) : 0ull;
      }
      sort128_desc(kk, lane);
      auto key_at = [&](int pos) -> u64 {  // the key at sorted position pos (warp-uniform)
        const int e = pos & 3;
        const u64 x = e == 0 ? kk[0] : e == 1 ? kk[1] : e == 2 ? kk[2] : kk[3];
        return __shfl_sync(FULL, x, pos >> 2);
      };
      const uint32_t tkey = (uint32_t)(key_at((int)k - 1) >> 32);
      tk = key2f(tkey);
      if (need_mass) {
        uint32_t q[4];
        expfx2(__fsub_rn(key2f((uint32_t)(kk[0] >> 32)), gmax), __fsub_rn(key2f((uint32_t)(kk[1] >> 32)), gmax), q[0],
               q[1]);
        expfx2(__fsub_rn(key2f((uint32_t)(kk[2] >> 32)), gmax), __fsub_rn(key2f((uint32_t)(kk[3] >> 32)), gmax), q[2],
               q[3]);
#pragma unroll
        for (int e = 0; e < 4; ++e) q[e] = (kk[e] != 0ull && (uint32_t)(kk[e] >> 32) >= tkey) ? q[e] : 0u;
        const u64 lsum = (u64)q[0] + q[1] + q[2] + q[3];
        const u64 incl = warp_incl_scan_u64(lsum, lane);
        qkept = __shfl_sync(FULL, incl, 31);
        int pcut = 128;
        if (dv.topp_on) {
          const double P = __dmul_rn((double)a.top_p, (double)qkept);
          const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
          u64 ab = incl - lsum;
          int my = -1;
          u64 myq = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (my < 0 && q[e] != 0u && ab <= plim && ab + q[e] > plim) {
              my = 4 * lane + e;
              myq = ab + q[e];
            }
            ab += q[e];
          }
          const unsigned bal = __ballot_sync(FULL, my >= 0);
          const int src = max(__ffs(bal) - 1, 0);
          pcut = max(__shfl_sync(FULL, my, src), 0);
          qkept = __shfl_sync(FULL, myq, src);
          const u64 ck = key_at(pcut), nk = key_at(min(pcut + 1, 127));
          cut_x = key2f((uint32_t)(ck >> 32));
          cut_id = (int32_t)(~(uint32_t)ck);
          topp_cut = true;
          if (pcut + 1 < 128 && nk != 0ull && (uint32_t)(nk >> 32) == (uint32_t)(ck >> 32)) status |= MTR_ROW_TIE_AT_CUT;
        }
        if (sel == MTR_SELECT_SAMPLE) {
          // the draw through 32 id buckets, as on the 64-key list
          const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
          bool kp[4];
          int ii[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            kp[e] = q[e] != 0u && 4 * lane + e <= pcut;
            ii[e] = (int)(~(uint32_t)kk[e]);
          }
          int bsh = 3;
          while ((32 << bsh) < VP) ++bsh;
          uint32_t* const bk = hc;
          *(uint2*)(bk + 2 * lane) = make_uint2(0u, 0u);
          __syncwarp();
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (kp[e]) {
              atomicAdd(bk + 2 * (ii[e] >> bsh), q[e] & 0xffffu);
              atomicAdd(bk + 2 * (ii[e] >> bsh) + 1, q[e] >> 16);
            }
          __syncwarp();
          const uint2 hh = *(const uint2*)(bk + 2 * lane);
          const u64 hb = ((u64)hh.y << 16) + hh.x;
          const u64 incl2 = warp_incl_scan_u64(hb, lane);
          const int b = max(__ffs(__ballot_sync(FULL, incl2 > R)) - 1, 0);
          const u64 f0 = __shfl_sync(FULL, incl2 - hb, b);
          u64 f[4] = {f0, f0, f0, f0};
          bool in[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) in[e] = kp[e] && (ii[e] >> bsh) == b;
#pragma unroll
          for (int e0 = 0; e0 < 4; ++e0) {
            unsigned mm = __ballot_sync(FULL, in[e0]);
#pragma unroll 1
            while (mm) {  // each entry of the bucket adds its mass to the entries at or above its id
              const int src = __ffs(mm) - 1;
              mm &= mm - 1u;
              const int is = __shfl_sync(FULL, ii[e0], src);
              const uint32_t qs = __shfl_sync(FULL, q[e0], src);
#pragma unroll
              for (int e = 0; e < 4; ++e) f[e] += is <= ii[e] ? qs : 0u;
            }
          }
          int32_t my = NO_ID;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (in[e] && f[e] > R && f[e] - q[e] <= R) my = min(my, ii[e]);
          token = __reduce_min_sync(FULL, my);
        }
      }
    } else if (need_mass && n >= 0) {
      // on the survivor list
#pragma unroll 1
      for (int j = lane; j < n; j += 32) lq[j] = expfx(__fsub_rn(lx[j], gmax));
      __syncwarp();
      u64 tot = 0;
#pragma unroll 1
      for (int j = lane; j < n; j += 32) tot += lq[j];
      tot = warp_sum_u64(tot);
      qkept = tot;
      // distance bins of the survivors (monotone in x): s3 spreads [0, d_max] over the bins
      float dmax = 0.0f;
#pragma unroll 1
      for (int j = lane; j < n; j += 32) dmax = fmaxf(dmax, __fsub_rn(gmax, lx[j]));
      dmax = __uint_as_float(__reduce_max_sync(FULL, __float_as_uint(dmax)));  // non-negative: bits order as floats
      const float s3 = dmax > 0.0f ? (float)(WNB - 1) / dmax : 0.0f;
      auto dbin3 = [&](float x) -> int {
        float z = __fmul_rn(__fsub_rn(gmax, x), s3);
        z = fminf(z, (float)(WNB - 1));
        return __float2int_rz(z);
      };
      if (dv.topp_on) {
        const double P = __dmul_rn((double)a.top_p, (double)tot);
        const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
#pragma unroll 1
        for (int i = lane * 2; i < WNB; i += 64) *(ulonglong2*)(hist + i) = make_ulonglong2(0ull, 0ull);
        __syncwarp();
        uint32_t* const hlo = (uint32_t*)hist;  // the 256 u64 bins as 256 low-half and 256 high-half sums
        uint32_t* const hhi = hlo + WNB;
#pragma unroll 1
        for (int j = lane; j < n; j += 32)
          if (lq[j]) {
            const int b = dbin3(lx[j]);
            atomicAdd(hlo + b, lq[j] & 0xffffu);
            atomicAdd(hhi + b, lq[j] >> 16);
          }
        __syncwarp();
        u64 above3, w3;
        const int b3 = max(warp_crossing_halves(hlo, hhi, plim, lane, above3, w3), 0);  // plim < total
        // canonical order (score desc, id asc) inside the crossing bin
        int m = 0;
#pragma unroll 1
        for (int j0 = 0; j0 < n; j0 += 32) {
          const int j = j0 + lane;
          const bool in = j < n && lq[j] != 0u && dbin3(lx[j]) == b3;
          const unsigned bm = __ballot_sync(FULL, in);
          const int pos = m + __popc(bm & ((1u << lane) - 1u));
          if (in && pos < WMINI) {
            mx[pos] = lx[j];
            mi[pos] = lid[j];
            mq[pos] = lq[j];
          }
          m += __popc(bm);
        }
        __syncwarp();
        float my_x = 0.0f;
        int32_t my_id = NO_ID;
        u64 my_q = 0;
        bool found = false;
        if (m <= WMINI) {
#pragma unroll 1
          for (int j = lane; j < m; j += 32) {
            const float xj = mx[j];
            const int32_t ij = mi[j];
            u64 am = above3;
#pragma unroll 1
            for (int jj = 0; jj < m; ++jj)
              if (canon_before(mx[jj], mi[jj], xj, ij)) am += mq[jj];
            if (am <= plim && am + mq[j] > plim) {
              my_x = xj;
              my_id = ij;
              my_q = am + mq[j];
              found = true;
            }
          }
        } else {
#pragma unroll 1
          for (int j = lane; j < n; j += 32) {
            const float xj = lx[j];
            const int32_t ij = lid[j];
            if (!lq[j]) continue;
            u64 am = 0;
#pragma unroll 1
            for (int jj = 0; jj < n; ++jj)
              if (canon_before(lx[jj], lid[jj], xj, ij)) am += lq[jj];
            if (am <= plim && am + lq[j] > plim) {
              my_x = xj;
              my_id = ij;
              my_q = am + lq[j];
              found = true;
            }
          }
        }
        const unsigned bf = __ballot_sync(FULL, found);
        const int src = max(__ffs(bf) - 1, 0);
        cut_x = __shfl_sync(FULL, my_x, src);
        cut_id = __shfl_sync(FULL, my_id, src);
        qkept = __shfl_sync(FULL, my_q, src);
        topp_cut = true;
        bool tie = false;
#pragma unroll 1
        for (int j = lane; j < n; j += 32) tie |= lx[j] == cut_x && lid[j] > cut_id;
        if (__any_sync(FULL, tie)) status |= MTR_ROW_TIE_AT_CUT;
        __syncwarp();
      }
      if (sel == MTR_SELECT_SAMPLE) {
        // id-ordered mass of the kept entries: id histogram, then the crossing bin
        const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
        int ish = 0;
        while ((VP >> ish) > WNB) ++ish;
#pragma unroll 1
        for (int i = lane * 2; i < WNB; i += 64) *(ulonglong2*)(hist + i) = make_ulonglong2(0ull, 0ull);
        __syncwarp();
        auto kept = [&](int j) -> bool {
          return lq[j] != 0u && (!topp_cut || lx[j] > cut_x || (lx[j] == cut_x && lid[j] <= cut_id));
        };
        uint32_t* const hlo = (uint32_t*)hist;  // low / high 16-bit sums, as above
        uint32_t* const hhi = hlo + WNB;
#pragma unroll 1
        for (int j = lane; j < n; j += 32)
          if (kept(j)) {
            atomicAdd(hlo + (lid[j] >> ish), lq[j] & 0xffffu);
            atomicAdd(hhi + (lid[j] >> ish), lq[j] >> 16);
          }
        __syncwarp();
        u64 above4, w4;
        const int b4 = max(warp_crossing_halves(hlo, hhi, R, lane, above4, w4), 0);  // R < qkept
        int m = 0;
#pragma unroll 1
        for (int j0 = 0; j0 < n; j0 += 32) {
          const int j = j0 + lane;
          const bool in = j < n && kept(j) && (lid[j] >> ish) == b4;
          const unsigned bm = __ballot_sync(FULL, in);
          const int pos = m + __popc(bm & ((1u << lane) - 1u));
          if (in && pos < WMINI) {
            mi[pos] = lid[j];
            mq[pos] = lq[j];
          }
          m += __popc(bm);
        }
        __syncwarp();
        int32_t my_tok = NO_ID;
        if (m <= WMINI) {
#pragma unroll 1
          for (int j = lane; j < m; j += 32) {
            const int32_t ij = mi[j];
            u64 cm2 = above4;
#pragma unroll 1
            for (int jj = 0; jj < m; ++jj)
              if (mi[jj] <= ij) cm2 += mq[jj];
            if (cm2 > R && cm2 - mq[j] <= R) my_tok = ij;
          }
        } else {
#pragma unroll 1
          for (int j = lane; j < n; j += 32) {
            if (!kept(j)) continue;
            const int32_t ij = lid[j];
            u64 cm2 = 0;
#pragma unroll 1
            for (int jj = 0; jj < n; ++jj)
              if (kept(jj) && lid[jj] <= ij) cm2 += lq[jj];
            if (cm2 > R && cm2 - lq[j] <= R) my_tok = ij;
          }
        }
        token = __reduce_min_sync(FULL, my_tok);
      }
    } else if (need_mass && !force_radix &&
               [&]() {
                 WDense dr;
                 warp_dense<SPLIT>(X, HALF, nch, V, gmax, tk, dv.topp_on != 0, a.top_p, a.top_p_mode,
                                   sel == MTR_SELECT_SAMPLE, u, (uint32_t*)hist, mx, mi, mq, lane, &dr);
                 if (!dr.ok) return false;
                 cut_x = dr.cut_x;
                 cut_id = dr.cut_id;
                 qkept = dr.qkept;
                 topp_cut = dr.topp_cut != 0;
                 status |= dr.status;
                 if (sel == MTR_SELECT_SAMPLE) token = dr.token;
                 return true;
               }()) {
      // the dense mass path (warp_dense) served the row
    } else if (need_mass) {
      // radix path over the whole row (no usable survivor list, or the dense path's
      // crossing bin held too many candidates)
      status |= MTR_ROW_SLOW_PATH;
      u64 tot = 0;
#pragma unroll 1
      for (int id = lane; id < V; id += 32) {
        const float x = *xat(id);
        if (finite_val(x) && x >= tk) tot += expfx(__fsub_rn(x, gmax));
      }
      tot = warp_sum_u64(tot);
      qkept = tot;
      if (dv.topp_on) {
        const double P = __dmul_rn((double)a.top_p, (double)tot);
        const u64 plim = a.top_p_mode == MTR_TOPP_HF ? __double2ull_rz(ceil(P)) - 1ull : __double2ull_rz(floor(P));
        uint32_t prefix = 0, mask = 0;
        u64 above = 0, lastw = 0;
#pragma unroll 1
        for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll 1
          for (int i = lane * 2; i < WNB; i += 64) *(ulonglong2*)(hist + i) = make_ulonglong2(0ull, 0ull);
          __syncwarp();
#pragma unroll 1
          for (int id = lane; id < V; id += 32) {
            const float x = *xat(id);
            if (finite_val(x) && x >= tk) {
              const uint32_t key = fkey(x);
              if ((key & mask) == prefix) {
                const uint32_t q = expfx(__fsub_rn(x, gmax));
                if (q) atomicAdd(hist + (255 - (int)((key >> shift) & 255u)), (u64)q);
              }
            }
          }
          __syncwarp();
          u64 ab;
          const int b = max(warp_crossing(hist, plim - above, lane, ab, lastw), 0);  // plim < total
          above += ab;
          prefix |= (255u - (uint32_t)b) << shift;
          mask |= 255u << shift;
          __syncwarp();
        }
        const float vstar = key2f(prefix);
        // the tie group at vstar shares one q
        uint32_t cnt_v = 0;
#pragma unroll 1
        for (int id = lane; id < V; id += 32) cnt_v += (*xat(id) == vstar);
        const uint32_t lastc = max(__reduce_add_sync(FULL, cnt_v), 1u);
        const u64 qv = max(lastw / (u64)lastc, 1ull);
        u64 nkeep = (plim - above) / qv + 1ull;
        if (nkeep > lastc) nkeep = lastc;
        cut_x = vstar;
        cut_id = NO_ID;
        if (nkeep < lastc) {
          // the nkeep-th smallest id of the tie group
          int32_t lo_id = -1;
          uint32_t seen = 0;
#pragma unroll 1
          for (int id0 = 0; id0 < V && seen < nkeep; id0 += 32) {
            const int id = id0 + lane;
            const bool hit = id < V && *xat(id) == vstar;
            const unsigned bm = __ballot_sync(FULL, hit);
            const uint32_t cb = __popc(bm);
            if (seen + cb >= nkeep) {
              unsigned mm = bm;
#pragma unroll 1
              for (uint32_t r = 1; r < nkeep - seen; ++r) mm &= mm - 1;
              lo_id = id0 + __ffs(mm) - 1;
            }
            seen += cb;
          }
          cut_id = lo_id;
          status |= MTR_ROW_TIE_AT_CUT;
        }
        qkept = above + nkeep * qv;
        topp_cut = true;
      }
      if (sel == MTR_SELECT_SAMPLE) {
        const u64 R = __double2ull_rz(floor(__dmul_rn((double)u, (double)qkept)));
        u64 run = 0;
        int32_t tok = -1;
#pragma unroll 1
        for (int id0 = 0; id0 < V && tok < 0; id0 += 32) {
          const int id = id0 + lane;
          u64 q = 0;
          if (id < V) {
            const float x = *xat(id);
            const bool kp = finite_val(x) && x >= tk && (!topp_cut || x > cut_x || (x == cut_x && id <= cut_id));
            q = kp ? expfx(__fsub_rn(x, gmax)) : 0u;
          }
          const u64 in = warp_incl_scan_u64(q, lane);
          const bool hit = q != 0 && run + in > R && run + in - q <= R;
          const unsigned bm = __ballot_sync(FULL, hit);
          if (bm) tok = id0 + __ffs(bm) - 1;
          run += __shfl_sync(FULL, in, 31);
        }
        token = tok;
      }
    }
    if (!clean && sel == MTR_SELECT_SAMPLE) token = (int32_t)a.pad_id;

    // ---------------------------------------------------------- processed scores / log-probs
    if (need_x_late) {
      const bool filter_out = clean && sel != MTR_SELECT_ARGMAX;
      double lse = 0.0;
      if (want_lp && clean) {
        if (!need_mass || sel == MTR_SELECT_ARGMAX) {
          u64 s = 0;
#pragma unroll 1
          for (int id = lane; id < V; id += 32) {
            const float x = *xat(id);
            s += finite_val(x) ? expfx(__fsub_rn(x, gmax)) : 0u;
          }
          qkept = warp_sum_u64(s);
        }
        lse = log((double)qkept) - 31.0 * 0.69314718055994530942;
      }
      float* srow = a.out_scores ? a.out_scores + row * a.out_scores_row_stride : nullptr;
      float* lrow = want_lp ? a.out_logprobs + row * a.out_logprobs_row_stride : nullptr;
#pragma unroll 1
      for (int i = lane * 4; i < V; i += 128) {
        const float4 f = *(const float4*)xat(i);
        const float v[4] = {f.x, f.y, f.z, f.w};
        float so[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool kp =
              !filter_out || (v[e] >= tk && (!topp_cut || v[e] > cut_x || (v[e] == cut_x && i + e <= cut_id)));
          so[e] = kp ? v[e] : NEG;
          lo[e] = !clean ? __int_as_float(0x7fc00000)
                         : (finite_val(v[e]) && kp) ? (float)(((double)v[e] - (double)gmax) - lse) : NEG;
        }
        if (srow) {
          if (dv.out_vec) {
            __stcs((float4*)(srow + i), make_float4(so[0], so[1], so[2], so[3]));
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (i + e < V) srow[i + e] = so[e];
          }
        }
        if (lrow) {
          if (dv.lp_vec) {
            __stcs((float4*)(lrow + i), make_float4(lo[0], lo[1], lo[2], lo[3]));
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (i + e < V) lrow[i + e] = lo[e];
          }
        }
      }
    }
    if (!issued) {
      issue_next();
      if (nrow < a.num_rows) load_ahead(a, dv, nrow, lane, L, ah);
    }
    if (lane == 0) {
      int32_t mm = mono;
      if (sel != MTR_SELECT_NONE) {
        const int64_t fin = finish_token(a, row, token, &status);
        if (a.flags & MTR_FLAG_MONO_UPDATE_FROM_SAMPLE) mm = mono_update(a, mm, fin);
        if ((a.flags & MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE) && a.prev_token) a.prev_token[row] = (int32_t)fin;
        if (a.out_ids) a.out_ids[row] = fin;
      }
      if (a.mono_mode != MTR_MONO_OFF && a.mono_state) a.mono_state[row] = mm;
      if (a.out_status) a.out_status[row] = status;
    }
    if (nrow < a.num_rows) load_ahead_class(a, lane, V, L, ah);  // the row-ahead values have landed by now
    __syncwarp();  // this row's readers of the shared regions are done
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Geo {
  int threads, ept, cs;
  int wide = 0;  // 256-thread CTAs, four per SM (more rows than one round of three holds)
};

// Up to one row per SM of a small vocabulary: one 512-thread CTA per row (8 ids
// per thread, the shortest per-row latency; 96-148 rows take 8.9-9.0 us where
// 256-thread CTAs took 10.2-10.5); otherwise one CTA (or cluster) per row.
static Geo pick_geo(int V, int64_t B, int sms) {
  if (V <= 4096) {
    if (B <= sms) return {512, 8, 1};
    return {256, 16, 1, B > 3 * (int64_t)sms ? 1 : 0};
  }
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

// SM count of the current device (148 when no device is visible, e.g. for
// geometry queries on a CPU-only host)
int device_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cache[dev] = n;
  }
  return cache[dev];
}

static thread_local int g_last_cuda_error = 0;
void set_last_cuda_error(int e) { g_last_cuda_error = e; }

static bool bad_float(float v) { return !(v == v) || v == INFINITY || v == -INFINITY; }

static int validate(const MtrSamplerArgs* a) {
  if (!a) return MTR_ERR_NULL_ARG;
  if (a->abi_version != MTR_ABI_VERSION || a->struct_size != sizeof(MtrSamplerArgs)) return MTR_ERR_ABI;
  const uint32_t kernel_flags = MTR_FLAG_KERNEL_ROW_CTA | MTR_FLAG_KERNEL_ROW_WARP | MTR_FLAG_KERNEL_STREAM;
  const uint32_t known = MTR_FLAG_MONO_UPDATE_FROM_IDS | MTR_FLAG_MONO_UPDATE_FROM_SAMPLE |
                         MTR_FLAG_GRAMMAR_PREV_FROM_IDS | MTR_FLAG_GRAMMAR_UPDATE_FROM_SAMPLE | MTR_FLAG_FORCE_RADIX |
                         kernel_flags | MTR_FLAG_TEST_COPY_TIMEOUT;
  if (a->flags & ~known) return MTR_ERR_BAD_PARAM;
  if (__builtin_popcount(a->flags & kernel_flags) > 1) return MTR_ERR_BAD_PARAM;
  if (a->num_rows < 0) return MTR_ERR_BAD_SHAPE;
  if (a->vocab < 1 || a->vocab > MTR_MAX_VOCAB) return MTR_ERR_BAD_SHAPE;
  if ((a->flags & MTR_FLAG_KERNEL_ROW_WARP) &&
      (a->vocab > WV_MAX || (a->input_ids && a->ids_len - a->penalty_start > WMAX_PEN_IDS)))
    return MTR_ERR_UNSUPPORTED;
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
    if ((uintptr_t)a->grammar_allow % 4 || (uintptr_t)a->grammar_vocab_bits % 4) return MTR_ERR_ALIGNMENT;
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
  // lookback bias
  if (a->lookback_mode < MTR_LOOKBACK_OFF || a->lookback_mode > MTR_LOOKBACK_RENORM) return MTR_ERR_BAD_PARAM;
  if (a->lookback_mode != MTR_LOOKBACK_OFF) {
    if (a->flags & (MTR_FLAG_KERNEL_ROW_WARP | MTR_FLAG_KERNEL_STREAM)) return MTR_ERR_UNSUPPORTED;
    if (a->lb_start < 0 || a->lb_end < a->lb_start || a->lb_end > a->vocab) return MTR_ERR_BAD_SHAPE;
  }
  // token append and stop counters
  if ((a->id_buffer || a->stop_counts) && a->select_mode == MTR_SELECT_NONE) return MTR_ERR_BAD_PARAM;
  if ((uintptr_t)a->stop_counts % 4) return MTR_ERR_ALIGNMENT;
  if (a->id_buffer) {
    if ((uintptr_t)a->id_buffer % 8 || (uintptr_t)a->cur_len_dev % 4) return MTR_ERR_ALIGNMENT;
    if (a->id_buffer_row_stride < 1) return MTR_ERR_BAD_SHAPE;
    if (!a->cur_len_dev && (a->cur_len < 0 || a->cur_len >= a->id_buffer_row_stride)) return MTR_ERR_BAD_SHAPE;
  }
  if (a->lookback_mode == MTR_LOOKBACK_RENORM) {
    if (a->lb_start >= a->vocab) return MTR_ERR_BAD_SHAPE;
    if (a->n_lb_eos < 0 || a->n_lb_eos > MTR_MAX_LB_EOS) return MTR_ERR_BAD_PARAM;
    for (int i = 0; i < a->n_lb_eos; ++i)
      if (a->lb_eos_ids[i] < 0 || a->lb_eos_ids[i] >= a->vocab) return MTR_ERR_BAD_PARAM;
    if (!a->lb_state || (a->ids_len > 0 && !a->lb_timed_bits)) return MTR_ERR_NULL_ARG;
    if ((uintptr_t)a->lb_state % 4 || (uintptr_t)a->lb_timed_bits % 4) return MTR_ERR_ALIGNMENT;
    if (a->ids_len > 0 && !a->input_ids) return MTR_ERR_NULL_ARG;
  }
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
  d.id_shift = 0;
  while (((a.vocab - 1) >> d.id_shift) >= NB) ++d.id_shift;
  d.gwords = (a.vocab + 31) / 32;
  d.temp_rcp = 1.0f / a.temperature;
  d.rep_rcp = (a.repetition_penalty >= 0x1p-30f && a.repetition_penalty <= 0x1p30f) ? 1.0f / a.repetition_penalty : 0.0f;
  d.neg_one = -1.0f;
  d.neg_zero = -0.0f;
  d.one = 1.0f;
  for (int c = 0; c < MTR_MAX_COND_TEMPS; ++c)
    d.cond_rcp[c] = (c < a.n_cond && a.cond_temperature[c] > 0.0f) ? 1.0f / a.cond_temperature[c] : 1.0f;
  for (int r = 0; r < MTR_MAX_COL_TEMP_RANGES; ++r)
    d.col_rcp[r] = (r < a.n_col_ranges && a.col_temperature[r] > 0.0f) ? 1.0f / a.col_temperature[r] : 1.0f;
  return d;
}

// The row-per-CTA kernel's opt-in to large dynamic shared memory, once per
// device and instantiation; it must precede any occupancy query of a launch
// whose shared memory passes 48 KB (the query reports 0 CTAs without it).
template <typename Tin, int TH, int EPT, int CS, int MINB = (TH <= 256 ? (CS == 1 ? 3 : 2) : 1)>
static cudaError_t cta_attr() {
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [&]() {
    const int max_dyn = 227 * 1024 - (int)sizeof(Shared<CS>);
    attr_err[dev] = cudaFuncSetAttribute(sampler_kernel<Tin, TH, EPT, CS, MINB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, max_dyn);
  });
  return attr_err[dev];
}

template <typename Tin, int TH, int EPT, int CS, int MINB = (TH <= 256 ? (CS == 1 ? 3 : 2) : 1)>
static cudaError_t launch_t(const MtrSamplerArgs& a, const Derived& d, int dyn, cudaStream_t s) {
  auto kern = sampler_kernel<Tin, TH, EPT, CS, MINB>;
  const cudaError_t ae = cta_attr<Tin, TH, EPT, CS, MINB>();
  if (ae != cudaSuccess) return ae;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(a.num_rows * CS), 1, 1);
  cfg.blockDim = dim3(TH, 1, 1);
  cfg.dynamicSmemBytes = (size_t)dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  cfg.numAttrs = launch_attrs(attr, CS, d.pdl != 0);
  cfg.attrs = cfg.numAttrs ? attr : nullptr;
  return cudaLaunchKernelEx(&cfg, kern, a, d);
}

// Occupancy of a kernel instantiation at a launch shape, per device, computed
// once and kept in a mutex-guarded table (threads launching different shapes
// never see a half-written entry).
cudaError_t cached_occupancy(const void* kern, int threads, int dyn, int* occ) {
  struct Ent {
    const void* k;
    int dev, threads, dyn, occ;
  };
  static std::mutex mu;
  static Ent tab[256];
  static int n = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < n; ++i)
      if (tab[i].k == kern && tab[i].dev == dev && tab[i].threads == threads && tab[i].dyn == dyn) {
        *occ = tab[i].occ;
        return cudaSuccess;
      }
  }
  int o = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, threads, (size_t)dyn);
  if (e != cudaSuccess) return e;
  if (o < 1) o = 1;
  std::lock_guard<std::mutex> lk(mu);
  if (n < 256) tab[n++] = Ent{kern, dev, threads, dyn, o};
  *occ = o;
  return cudaSuccess;
}

// Kernel choice.  Vocabularies above 4096 with a top-k in [1, 64] take the
// streaming row-group kernel (several warps per row, no staged row: 2-8x the
// row-per-CTA kernel there).  For V <= 4096 the row-per-warp kernel wins when
// many rows each end in a short list (argmax, or top-k with k <=
// WARP_TOPK_MAX) and more rows than one round of row-per-CTA CTAs holds.
// Everything else (top-p over the whole row, column temperatures, rows that fit
// one round of CTAs) takes the row-per-CTA kernel.  The flags force a kernel.
constexpr int WARP_TOPK_MAX = 128;
enum { KERNEL_ROW_CTA = 0, KERNEL_ROW_WARP = 1, KERNEL_STREAM = 2 };

template <typename Tin>
static const void* cta256_ptr() {
  if (cta_attr<Tin, 256, 16, 1>() != cudaSuccess) return nullptr;
  return (const void*)sampler_kernel<Tin, 256, 16, 1>;
}
// Rows that one round of row-per-CTA CTAs holds at a V <= 4096 launch (one
// 512-thread CTA per SM up to #SMs rows, else the 256-thread CTAs' occupancy:
// 3 per SM, penalty tiles included).  Within one round the row-per-CTA kernel beats the row-per-warp
// kernel (sharded chain, 296-440 pairs: 14.1-14.5 us against 15.6-16.0).
static int64_t cta_round_rows(const MtrSamplerArgs& a, const Derived& d, int sms) {
  if (a.num_rows <= sms) return sms;
  const Geo g = pick_geo(a.vocab, a.num_rows, sms);
  const void* k = a.logits_dtype == MTR_DTYPE_F32    ? cta256_ptr<float>()
                  : a.logits_dtype == MTR_DTYPE_BF16 ? cta256_ptr<__nv_bfloat16>()
                                                     : cta256_ptr<__half>();
  int occ = 0;
  if (!k || cached_occupancy(k, g.threads, dyn_smem_bytes(g, d.pen_on != 0), &occ) != cudaSuccess) {
    cudaGetLastError();
    occ = 3;  // no device: the launch bound
  }
  return (int64_t)occ * sms;
}

static int pick_kernel(const MtrSamplerArgs& a, const Derived& d, int sms) {
  if (a.flags & MTR_FLAG_KERNEL_ROW_CTA) return KERNEL_ROW_CTA;
  if (a.flags & MTR_FLAG_KERNEL_ROW_WARP) return KERNEL_ROW_WARP;
  if (a.flags & MTR_FLAG_KERNEL_STREAM) return KERNEL_STREAM;
  if (a.lookback_mode != MTR_LOOKBACK_OFF) return KERNEL_ROW_CTA;  // the lookback bias lives in the row-per-CTA kernel
  if (a.vocab > WV_MAX && sk_supported(a, d)) return KERNEL_STREAM;
  if (a.vocab > WV_MAX || a.num_rows <= cta_round_rows(a, d, sms)) return KERNEL_ROW_CTA;
  if (d.pen_on && a.ids_len - a.penalty_start > WMAX_PEN_IDS) return KERNEL_ROW_CTA;
  // top-p over the whole row stays on the row-per-CTA kernel: a warp's dense
  // path (warp_dense) is latency-bound on a full row of exponentials
  const bool short_list = a.select_mode == MTR_SELECT_ARGMAX || (d.topk_on && a.top_k <= WARP_TOPK_MAX);
  return short_list ? KERNEL_ROW_WARP : KERNEL_ROW_CTA;
}

// Host checks plus the kernel a flag forces: MTR_ERR_UNSUPPORTED when the
// request does not fit it.
static int validate_all(const MtrSamplerArgs* a) {
  const int v = validate(a);
  if (v != MTR_OK) return v;
  if ((a->flags & MTR_FLAG_KERNEL_STREAM) && a->num_rows > 0 && !sk_supported(*a, derive(*a))) return MTR_ERR_UNSUPPORTED;
  return MTR_OK;
}

template <typename Tin, bool CFG>
static const void* warp_kernel_ptr() {
  return (const void*)row_warp_kernel<Tin, CFG>;
}
static const void* warp_kernel_for(const MtrSamplerArgs& a) {
  const bool cfg = a.cfg_enabled != 0;
  switch (a.logits_dtype) {
    case MTR_DTYPE_F32: return cfg ? warp_kernel_ptr<float, true>() : warp_kernel_ptr<float, false>();
    case MTR_DTYPE_BF16: return cfg ? warp_kernel_ptr<__nv_bfloat16, true>() : warp_kernel_ptr<__nv_bfloat16, false>();
    default: return cfg ? warp_kernel_ptr<__half, true>() : warp_kernel_ptr<__half, false>();
  }
}

// Persistent grid: as many one-warp CTAs as fit on the device (each walks rows
// r, r + grid, ... and prefetches its next row into L2), at most one per row.
template <typename Tin, bool CFG>
static cudaError_t launch_warp_t(const MtrSamplerArgs& a, const Derived& d, cudaStream_t s) {
  auto kern = row_warp_kernel<Tin, CFG>;
  const int dyn = warp_bytes(a.vocab);
  int occ = 0;
  cudaError_t e = cached_occupancy((const void*)kern, 32, dyn, &occ);
  if (e != cudaSuccess) return e;
  const int64_t cap = (int64_t)occ * device_sms();
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3((unsigned)(a.num_rows < cap ? a.num_rows : cap), 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.dynamicSmemBytes = (size_t)dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  cfg.numAttrs = launch_attrs(attr, 1, d.pdl != 0);
  cfg.attrs = cfg.numAttrs ? attr : nullptr;
  return cudaLaunchKernelEx(&cfg, kern, a, d);
}
template <typename Tin>
static cudaError_t launch_warp(const MtrSamplerArgs& a, const Derived& d, cudaStream_t s) {
  return a.cfg_enabled ? launch_warp_t<Tin, true>(a, d, s) : launch_warp_t<Tin, false>(a, d, s);
}

template <typename Tin>
static cudaError_t launch_dtype(const MtrSamplerArgs& a, const Derived& d, const Geo& g, int dyn, cudaStream_t s) {
  if (g.threads == 512 && g.ept == 8 && g.cs == 1) return launch_t<Tin, 512, 8, 1>(a, d, dyn, s);
  if (g.threads == 256 && g.cs == 1)
    return g.wide ? launch_t<Tin, 256, 16, 1, 4>(a, d, dyn, s) : launch_t<Tin, 256, 16, 1>(a, d, dyn, s);
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

int mtr_sampler_validate(const MtrSamplerArgs* a) { return mtr::validate_all(a); }

int mtr_sampler_query(int32_t vocab, int32_t num_rows, int32_t with_penalties, MtrLaunchInfo* out) {
  if (!out) return MTR_ERR_NULL_ARG;
  if (vocab < 1 || vocab > MTR_MAX_VOCAB || num_rows < 0) return MTR_ERR_BAD_SHAPE;
  const mtr::Geo g = mtr::pick_geo(vocab, num_rows, mtr::device_sms());
  out->threads = g.threads;
  out->elems_per_thread = g.ept;
  out->cluster_size = g.cs;
  out->grid = num_rows * g.cs;
  out->dyn_smem_bytes = mtr::dyn_smem_bytes(g, with_penalties != 0);
  out->max_vocab = MTR_MAX_VOCAB;
  out->max_ids_len = MTR_MAX_IDS_LEN;
  out->candidate_cap = mtr::CAP;
  out->kernel = mtr::KERNEL_ROW_CTA;
  return MTR_OK;
}

int mtr_sampler_query_args(const MtrSamplerArgs* a, MtrLaunchInfo* out) {
  if (!out) return MTR_ERR_NULL_ARG;
  const int v = mtr::validate_all(a);
  if (v != MTR_OK) return v;
  const mtr::Derived d = mtr::derive(*a);
  const int sms = mtr::device_sms();
  const int k = mtr::pick_kernel(*a, d, sms);
  out->max_vocab = MTR_MAX_VOCAB;
  out->max_ids_len = MTR_MAX_IDS_LEN;
  out->cluster_size = 1;
  if (k == mtr::KERNEL_STREAM) {
    mtr::stream_query(*a, d, sms, out);
    return MTR_OK;
  }
  if (k == mtr::KERNEL_ROW_WARP) {
    out->threads = 32;
    out->elems_per_thread = mtr::warp_vpad(a->vocab) / 32;
    int occ = 0;
    const int dyn = mtr::warp_bytes(a->vocab);
    if (mtr::cached_occupancy(mtr::warp_kernel_for(*a), 32, dyn, &occ) != cudaSuccess) {
      cudaGetLastError();
      occ = 10;  // no device: the launch bound
    }
    const int64_t cap = (int64_t)occ * sms;
    out->grid = (int32_t)(a->num_rows < cap ? a->num_rows : cap);
    out->dyn_smem_bytes = dyn;
    out->candidate_cap = mtr::WCAP;
    out->kernel = mtr::KERNEL_ROW_WARP;
    return MTR_OK;
  }
  return mtr_sampler_query(a->vocab, a->num_rows, d.pen_on, out);
}

int mtr_sampler_launch(const MtrSamplerArgs* a, void* stream) {
  const int v = mtr::validate_all(a);
  if (v != MTR_OK) return v;
  if (a->num_rows == 0) return MTR_OK;
  return mtr::sampler_launch(a, (cudaStream_t)stream, true);
}

}  // extern "C"

int mtr::sampler_launch(const MtrSamplerArgs* a, cudaStream_t s, bool pdl) {
  mtr::Derived d = mtr::derive(*a);
  d.pdl = pdl ? 1 : 0;
  const int sms = mtr::device_sms();
  cudaError_t e;
  const int k = mtr::pick_kernel(*a, d, sms);
  if (k == mtr::KERNEL_STREAM) {
    e = mtr::stream_launch(*a, d, sms, s);
  } else if (k == mtr::KERNEL_ROW_WARP) {
    switch (a->logits_dtype) {
      case MTR_DTYPE_F32: e = mtr::launch_warp<float>(*a, d, s); break;
      case MTR_DTYPE_BF16: e = mtr::launch_warp<__nv_bfloat16>(*a, d, s); break;
      default: e = mtr::launch_warp<__half>(*a, d, s); break;
    }
  } else {
    const mtr::Geo g = mtr::pick_geo(a->vocab, a->num_rows, sms);
    const int dyn = mtr::dyn_smem_bytes(g, d.pen_on != 0);
    switch (a->logits_dtype) {
      case MTR_DTYPE_F32: e = mtr::launch_dtype<float>(*a, d, g, dyn, s); break;
      case MTR_DTYPE_BF16: e = mtr::launch_dtype<__nv_bfloat16>(*a, d, g, dyn, s); break;
      default: e = mtr::launch_dtype<__half>(*a, d, g, dyn, s); break;
    }
  }
  mtr::g_last_cuda_error = (int)e;
  return e == cudaSuccess ? MTR_OK : MTR_ERR_CUDA;
}

extern "C" {

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
