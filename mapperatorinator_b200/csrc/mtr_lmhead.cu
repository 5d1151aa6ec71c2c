// mtr_lmhead.cu -- the decoder's output projection on the sm_100a tensor cores,
// feeding the fused sampler.
//
// logits[R, V] = RN_bf16(hidden[R, d] . weight[V, d]^T), fp32 accumulation:
// VarWhisperForConditionalGeneration.proj_out, an nn.Linear(d_model, vocab,
// bias=False) run in the model's bf16 dtype
// (osuT5/osuT5/model/custom_transformers/modeling_varwhisper.py:1583, 1647-1649),
// whose bf16 output the decode loops turn into fp32 scores
// (optimized/single/decode_loop.py:290-294).
//
// One CTA owns a BM x BN tile of logits (BM = 128 rows, BN = 64 or 128 vocabulary
// ids) and walks d in BK = 64 steps:
//   warp 0, one lane   TMA producer: 2-D tiled loads (128-byte swizzle) of the
//                      hidden and weight tiles into a STAGES-deep shared ring,
//                      completion counted on a per-stage mbarrier
//   warp 1, one lane   MMA issuer: four tcgen05.mma.cta_group::1.kind::f16
//                      (M=128, N=BN, K=16, bf16 x bf16 -> fp32) per stage, the
//                      accumulator in tensor memory; tcgen05.commit frees the
//                      stage and finally signals the epilogue
//   warp 2             allocates / frees the BN tensor-memory columns
//   warps 0-3          epilogue: tcgen05.ld of the accumulator rows (warp w owns
//                      TMEM lanes 32w..32w+31 = tile rows), bf16 round to
//                      nearest even, 16-byte stores of the logits row segments
// Every mbarrier wait is bounded; a wait that gives up raises the error word and
// the CTA stops issuing, drains what it started (bounded again), frees its tensor
// memory and returns.  No cluster launch and no multicast: every load reads this
// GPU's own memory into this CTA's shared memory.
//
// The sampler needs whole rows while a tile holds BN columns of 128 rows, and a
// row of tensor memory holds at most 512 fp32 columns, so the logits of one step
// meet the sampler in L2 (R x V x 2 bytes, 2 MiB for 256 x 4096): the sampler
// launch that follows uses programmatic dependent launch and waits for this
// grid at griddepcontrol.wait.  This kernel lets its dependents in only as its
// CTAs exit (no early launch_dependents): admitted during the epilogue, the
// sampler's CTAs crowded onto the few SMs without a 150 KB projection CTA and
// the pair took 1.9 us longer.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "mtr_common.cuh"

namespace mtr {
namespace lm {

constexpr int BM = 128;
constexpr int BK = 64;  // bf16 elements per 128-byte swizzled row
constexpr int UK = 16;  // K of one tcgen05.mma kind::f16
constexpr uint64_t WAIT_NS = 200000000ull;  // 200 ms: far beyond any healthy wait

struct Params {
  __nv_bfloat16* out;
  int64_t out_stride;
  int32_t rows;
  int32_t vocab;
  int32_t kblocks;
  uint32_t* err;
};

// ---------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase with parity `ph` to complete; false after `budget_ns`
// nanoseconds (0: a single poll).  The clock is read only every 4096 polls:
// a healthy hand-off completes long before the first read.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t ph, uint64_t budget_ns) {
  const uint32_t a = smem_u32(b);
  uint64_t t0 = 0;
  for (uint32_t i = 1;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(ph)
        : "memory");
    if (done) return true;
    if (budget_ns == 0) return false;
    if ((i & 4095u) == 0u) {
      const uint64_t t = global_ns();
      if (t0 == 0) t0 = t;
      else if (t - t0 > budget_ns) return false;
    }
  }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with the 128-byte swizzle:
// rows of 128 bytes, 8-row atoms 1024 bytes apart (stride byte offset), leading
// byte offset 16 (unused by this layout), descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4-5 = 1), bf16 A
// and B (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <int N>
__host__ __device__ constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <int BN>
struct Ring {
  static constexpr int STAGES = BN == 64 ? 6 : 4;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
};

template <int BN>
__global__ void __launch_bounds__(128, 1)
    lmhead_gemm_kernel(const __grid_constant__ CUtensorMap map_h, const __grid_constant__ CUtensorMap map_w,
                       const Params p) {
  using RG = Ring<BN>;
  constexpr int S = RG::STAGES;
  extern __shared__ uint8_t dsm_raw[];
  __shared__ __align__(8) uint64_t full[S], empty[S], done;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile uint32_t abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  // 1024-byte aligned ring (the 128-byte swizzle pattern repeats every 8 rows)
  const uint32_t raw = smem_u32(dsm_raw);
  uint8_t* ring = dsm_raw + (((raw + 1023u) & ~1023u) - raw);
  auto a_tile = [&](int s) { return ring + (size_t)s * RG::STAGE_BYTES; };
  auto b_tile = [&](int s) { return ring + (size_t)s * RG::STAGE_BYTES + RG::A_BYTES; };

  // the producer (thread 0) initialises the barriers and issues the first ring
  // stages at once: the loads need no tensor memory, so they overlap its
  // allocation and the setup barrier
  const int KB = p.kblocks;
  const int first = KB < S ? KB : S;
  if (threadIdx.x == 0) {
    // the descriptors first, then the barriers; launched as a programmatic
    // dependent, the CTA reaches here while the previous kernel drains, and
    // waits for it (griddepcontrol.wait) before its first global access
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_h) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&map_w) : "memory");
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    wait_prior_grid();
    for (int kb = 0; kb < first; ++kb) {
      mbar_expect_tx(&full[kb], RG::STAGE_BYTES);
      tma_load_2d(a_tile(kb), &map_h, kb * BK, m0, &full[kb]);
      tma_load_2d(b_tile(kb), &map_w, kb * BK, n0, &full[kb]);
    }
  }
  if (warp == 2) {  // the whole warp allocates; BN is a power of two >= 32
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"((uint32_t)BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  wait_prior_grid();  // every thread: its logits stores follow the previous kernel's reads
  const uint32_t tmem = tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- producer (the first `first` stages are in flight already)
    int issued = first;
    for (int kb = first; kb < KB; ++kb) {
      const int s = kb % S;
      if (kb >= S && !mbar_wait(&empty[s], ((kb / S) & 1) ^ 1, WAIT_NS)) {
        abort_flag = 1u;
        if (p.err) atomicOr(p.err, 1u);
        break;
      }
      if (abort_flag) break;
      mbar_expect_tx(&full[s], RG::STAGE_BYTES);
      tma_load_2d(a_tile(s), &map_h, kb * BK, m0, &full[s]);
      tma_load_2d(b_tile(s), &map_w, kb * BK, n0, &full[s]);
      issued = kb + 1;
    }
    // copies still in flight land before the CTA may leave (bounded)
    for (int kb = (issued > S ? issued - S : 0); kb < issued; ++kb)
      mbar_wait(&full[kb % S], (kb / S) & 1, abort_flag ? WAIT_NS : 0ull);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = idesc_bf16<BN>();
    bool ok = true;
    for (int kb = 0; kb < KB && ok; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(&full[s], (kb / S) & 1, WAIT_NS) || abort_flag) {
        abort_flag = 1u;
        if (p.err) atomicOr(p.err, 2u);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_u32(a_tile(s)), b0 = smem_u32(b_tile(s));
#pragma unroll
      for (int k = 0; k < BK / UK; ++k)
        tc_mma(tmem, sw128_desc(a0 + k * UK * 2), sw128_desc(b0 + k * UK * 2), idesc, (kb | k) != 0 ? 1u : 0u);
      tc_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    tc_commit(&done);  // arrives when every MMA issued above has completed
  }
  __syncwarp();

  // ---------------- epilogue: all four warps; one lane per warp polls the
  // barrier (128 pollers would contend with the copies' completions for it)
  bool waited = true;
  if (lane == 0) waited = mbar_wait(&done, 0, WAIT_NS);
  waited = __shfl_sync(FULL, waited, 0) != 0;
  tc_fence_after();
  // tcgen05.ld is warp-collective: the whole warp reads or none of it
  const bool go = __all_sync(FULL, waited && !abort_flag);
  if (!waited && lane == 0 && p.err) atomicOr(p.err, 4u);
  if (go) {
    const int row = m0 + warp * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
          "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
          "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
            "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
            "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
          : "r"(lane_base + (uint32_t)(c * 32)));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(v[2 * j]), __uint_as_float(v[2 * j + 1]));
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
      const int col = n0 + c * 32;
      if (row < p.rows) {
        __nv_bfloat16* dst = p.out + (int64_t)row * p.out_stride + col;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (col + 8 * q < p.vocab) *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BN) : "memory");
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)f;
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix (cols contiguous),
// box of BK columns x box_rows rows, 128-byte swizzle, out-of-range rows read 0.
static bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t row_stride, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(row_stride * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int pick_tile_n(const MtrLmHeadArgs& a, int sms) {
  if (a.tile_n) return a.tile_n;
  const int64_t mt = (a.rows + BM - 1) / BM;
  // the wider tile when it still gives every SM a CTA, else twice the CTAs
  return mt * ((a.vocab + 127) / 128) >= sms ? 128 : 64;
}

template <int BN>
static cudaError_t launch_bn(const MtrLmHeadArgs& a, cudaStream_t s) {
  CUtensorMap mh, mw;
  if (!make_map(&mh, a.hidden, a.rows, a.d_model, a.hidden_row_stride, BM) ||
      !make_map(&mw, a.weight, a.vocab, a.d_model, a.weight_row_stride, BN))
    return cudaErrorInvalidValue;
  auto kern = lmhead_gemm_kernel<BN>;
  static std::once_flag once[64];
  static cudaError_t attr_err[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [&]() {
    attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Ring<BN>::BYTES);
  });
  if (attr_err[dev] != cudaSuccess) return attr_err[dev];
  Params p;
  p.out = (__nv_bfloat16*)a.logits;
  p.out_stride = a.logits_row_stride;
  p.rows = a.rows;
  p.vocab = a.vocab;
  p.kblocks = a.d_model / BK;
  p.err = a.error_word;
  const dim3 grid((unsigned)((a.vocab + BN - 1) / BN), (unsigned)((a.rows + BM - 1) / BM), 1);
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = Ring<BN>::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  cfg.numAttrs = launch_attrs(attr, 1, true);
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kern, mh, mw, p);
}

}  // namespace lm
}  // namespace mtr

// ---------------------------------------------------------------- C ABI
int mtr_lmhead_validate(const MtrLmHeadArgs* a) {
  if (!a) return MTR_ERR_NULL_ARG;
  if (a->abi_version != MTR_ABI_VERSION || a->struct_size != sizeof(MtrLmHeadArgs)) return MTR_ERR_ABI;
  if (a->rows < 0) return MTR_ERR_BAD_SHAPE;
  if (a->d_model < mtr::lm::BK || a->d_model % mtr::lm::BK) return MTR_ERR_BAD_SHAPE;
  if (a->vocab < 8 || a->vocab % 8 || a->vocab > MTR_MAX_VOCAB) return MTR_ERR_BAD_SHAPE;
  if (a->tile_n != 0 && a->tile_n != 64 && a->tile_n != 128) return MTR_ERR_BAD_PARAM;
  if (a->rows == 0) return MTR_OK;
  if (!a->hidden || !a->weight || !a->logits) return MTR_ERR_NULL_ARG;
  if ((uintptr_t)a->hidden % 16 || (uintptr_t)a->weight % 16 || (uintptr_t)a->logits % 16 ||
      (uintptr_t)a->error_word % 4)
    return MTR_ERR_ALIGNMENT;
  if (a->hidden_row_stride < a->d_model || a->weight_row_stride < a->d_model || a->logits_row_stride < a->vocab)
    return MTR_ERR_BAD_SHAPE;
  if (a->hidden_row_stride % 8 || a->weight_row_stride % 8 || a->logits_row_stride % 8) return MTR_ERR_ALIGNMENT;
  return MTR_OK;
}

static int lmhead_launch_impl(const MtrLmHeadArgs* a, cudaStream_t s) {
  const int sms = mtr::device_sms();
  const int bn = mtr::lm::pick_tile_n(*a, sms);
  const cudaError_t e = bn == 64 ? mtr::lm::launch_bn<64>(*a, s) : mtr::lm::launch_bn<128>(*a, s);
  mtr::set_last_cuda_error((int)e);
  return e == cudaSuccess ? MTR_OK : MTR_ERR_CUDA;
}

int mtr_lmhead_launch(const MtrLmHeadArgs* a, void* stream) {
  const int v = mtr_lmhead_validate(a);
  if (v != MTR_OK) return v;
  if (a->rows == 0) return MTR_OK;
  return lmhead_launch_impl(a, (cudaStream_t)stream);
}

int mtr_lmhead_sample_launch(const MtrLmHeadArgs* lm, const MtrSamplerArgs* sa, void* stream) {
  int v = mtr_lmhead_validate(lm);
  if (v != MTR_OK) return v;
  v = mtr_sampler_validate(sa);
  if (v != MTR_OK) return v;
  // the sampler reads exactly the logits the GEMM writes
  if (sa->logits != lm->logits || sa->logits_dtype != MTR_DTYPE_BF16 || sa->logits_row_stride != lm->logits_row_stride ||
      sa->vocab != lm->vocab)
    return MTR_ERR_BAD_PARAM;
  const int64_t second = sa->cfg_second_offset > 0 ? sa->cfg_second_offset : sa->num_rows;
  const int64_t need = sa->cfg_enabled ? second + sa->num_rows : sa->num_rows;
  if (need > lm->rows) return MTR_ERR_BAD_SHAPE;
  if (lm->rows == 0 || sa->num_rows == 0) return MTR_OK;
  cudaStream_t s = (cudaStream_t)stream;
  v = lmhead_launch_impl(lm, s);
  if (v != MTR_OK) return v;
  return mtr::sampler_launch(sa, s, true);
}
