// Kernel instantiations for one GGUF format (one translation unit per format
// so the build compiles formats in parallel).
#include "launch.cuh"

namespace frc {
template cudaError_t launch_gemv<kQ8_0>(const GemvRequest&);
template cudaError_t launch_dequant<kQ8_0>(const DequantRequest&);
template cudaError_t launch_gemm_tc<kQ8_0>(const GemvRequest&);
}  // namespace frc
