// mtr_stream_f32.cu -- the streaming row-group kernel instantiated for float logits.
#include "mtr_stream.cuh"

namespace mtr {

MTR_STREAM_INSTANTIATE(float, f32)

}  // namespace mtr
