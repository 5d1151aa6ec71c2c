// mtr_stream_f16.cu -- the streaming row-group kernel instantiated for __half logits.
#include "mtr_stream.cuh"

namespace mtr {

MTR_STREAM_INSTANTIATE(__half, f16)

}  // namespace mtr
