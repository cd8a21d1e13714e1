#include "gemm.cuh"
namespace zc {
int gemm_f32_device(const float *, const float *, float *, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                    bool, bool, const GemmBatch &, int64_t, cudaStream_t) {
    return set_error(ZPUCUDA_ERR_NOT_SUPPORTED, "f32 gemm kernel not built yet");
}
}  // namespace zc
