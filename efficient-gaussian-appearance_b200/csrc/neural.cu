// Neural appearance (placeholder until the tensor-core MLP lands).
#include "launch.h"

namespace fgs {

cudaError_t launch_preprocess_fwd_neural(const Params&, const AppearanceConfig&, const View&, const PrimBuffers&, cudaStream_t) {
    return cudaErrorNotSupported;
}
cudaError_t launch_preprocess_bwd_neural(const Params&, const AppearanceConfig&, const View&, const uint32_t*, const Record*,
                                         const GradRecord*, const GradOut&, cudaStream_t) {
    return cudaErrorNotSupported;
}
size_t neural_grad_scratch_floats(const AppearanceConfig& A) { return static_cast<size_t>(A.n_params); }

}  // namespace fgs
