// attention_f32.cu -- the F32 instances of the decode-attention kernel
// (compiled apart so the three element types build in parallel).
#include "attention.cuh"

namespace ane {
template int launch_decode_attention<F32>(const AttnArgs&, int, int, int64_t, cudaStream_t);
}  // namespace ane
