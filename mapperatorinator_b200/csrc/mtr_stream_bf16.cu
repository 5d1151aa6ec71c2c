// mtr_stream_bf16.cu -- the streaming row-group kernel instantiated for __nv_bfloat16 logits.
#include "mtr_stream.cuh"

namespace mtr {

MTR_STREAM_INSTANTIATE(__nv_bfloat16, bf16)

}  // namespace mtr
