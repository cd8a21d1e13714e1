// rng.Rng on the device (src/zpu/rng.zig:15-102).  splitmix64's state after
// i draws is seed + i * gamma, so draw i is a pure function of (seed, i) and
// every element can be generated independently: the stream is the same one
// zpu's sequential generator produces.
#include "common.cuh"

namespace zc {

__device__ __forceinline__ uint64_t splitmix_at(uint64_t seed, uint64_t draw /* 1-based */) {
    uint64_t z = seed + draw * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
__device__ __forceinline__ double u01_at(uint64_t seed, uint64_t draw) {
    return (double)(splitmix_at(seed, draw) >> 11) * (1.0 / 9007199254740992.0);
}

// Rng.uniformRange (rng.zig:46-51): element i uses draw i + 1.
template <class T>
__global__ void uniform_kernel(uint64_t seed, T *out, int64_t n, double lo, double hi) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (T)(lo + (hi - lo) * u01_at(seed, (uint64_t)i + 1));
}

// Rng.normal (rng.zig:54-71): pair j uses draws 2j+1, 2j+2 and writes
// elements 2j (r cos) and 2j+1 (r sin).
template <class T>
__global__ void normal_kernel(uint64_t seed, T *out, int64_t n) {
    const int64_t pairs = (n + 1) / 2;
    for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < pairs; j += (int64_t)gridDim.x * blockDim.x) {
        double a1 = u01_at(seed, 2 * (uint64_t)j + 1);
        if (a1 < 1e-12) a1 = 1e-12;
        const double a2 = u01_at(seed, 2 * (uint64_t)j + 2);
        const double r = sqrt(-2.0 * log(a1));
        const double th = 6.283185307179586 * a2;
        double s, c;
        sincos(th, &s, &c);
        out[2 * j] = (T)(r * c);
        if (2 * j + 1 < n) out[2 * j + 1] = (T)(r * s);
    }
}

// Rng.randint (rng.zig:93-101).
__global__ void randint_kernel(uint64_t seed, int64_t *out, int64_t n, int64_t lo, uint64_t span) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = lo + (int64_t)(splitmix_at(seed, (uint64_t)i + 1) % span);
}

static int grid_for(int64_t n) {
    int64_t g = (n + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 16;
    return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace zc

using namespace zc;

extern "C" {

int zpucuda_rng_uniform(uint64_t seed, int dtype, void *d_out, int64_t n, double lo, double hi, void *stream) {
    ZC_CHECK(n >= 0 && (d_out || !n), ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (!n) return ZPUCUDA_OK;
    cudaStream_t s = resolve_stream(stream);
    if (dtype == ZPUCUDA_F32) uniform_kernel<float><<<grid_for(n), 256, 0, s>>>(seed, (float *)d_out, n, lo, hi);
    else if (dtype == ZPUCUDA_F64) uniform_kernel<double><<<grid_for(n), 256, 0, s>>>(seed, (double *)d_out, n, lo, hi);
    else return ZPUCUDA_ERR_NOT_SUPPORTED;
    ZC_LAUNCHED("uniform_kernel");
    return ZPUCUDA_OK;
}

int zpucuda_rng_normal(uint64_t seed, int dtype, void *d_out, int64_t n, void *stream) {
    ZC_CHECK(n >= 0 && (d_out || !n), ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (!n) return ZPUCUDA_OK;
    cudaStream_t s = resolve_stream(stream);
    const int64_t pairs = (n + 1) / 2;
    if (dtype == ZPUCUDA_F32) normal_kernel<float><<<grid_for(pairs), 256, 0, s>>>(seed, (float *)d_out, n);
    else if (dtype == ZPUCUDA_F64) normal_kernel<double><<<grid_for(pairs), 256, 0, s>>>(seed, (double *)d_out, n);
    else return ZPUCUDA_ERR_NOT_SUPPORTED;
    ZC_LAUNCHED("normal_kernel");
    return ZPUCUDA_OK;
}

int zpucuda_rng_randint(uint64_t seed, int64_t *d_out, int64_t n, int64_t lo, int64_t hi, void *stream) {
    ZC_CHECK(n >= 0 && (d_out || !n), ZPUCUDA_ERR_INVALID_ARGUMENT);
    if (hi <= lo) return ZPUCUDA_ERR_SHAPE_MISMATCH;  // rng.zig:94
    if (!n) return ZPUCUDA_OK;
    cudaStream_t s = resolve_stream(stream);
    randint_kernel<<<grid_for(n), 256, 0, s>>>(seed, d_out, n, lo, (uint64_t)(hi - lo));
    ZC_LAUNCHED("randint_kernel");
    return ZPUCUDA_OK;
}

}  // extern "C"
