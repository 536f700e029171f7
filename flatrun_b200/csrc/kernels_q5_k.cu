// Kernel instantiations for one GGUF format (one translation unit per format
// so the build compiles formats in parallel).
#include "launch.cuh"

namespace frc {
template cudaError_t launch_gemv<kQ5_K>(const GemvRequest&);
template cudaError_t launch_dequant<kQ5_K>(const DequantRequest&);
template cudaError_t launch_gemm_tc<kQ5_K>(const GemvRequest&);
}  // namespace frc
