// Seeded synthetic data: the random-init weights of the QW3M blob and
// synthetic token ids, generated on the device.
//
// u64(seed, stream, i) = splitmix64(key + i * 0xD1B54A32D192ED03),
//   key = splitmix64(seed ^ splitmix64(stream)).
// normal(sigma): the four 16-bit lanes of u64 summed (Irwin-Hall, n = 4),
//   centred, times the FP32 constant sigma * sqrt(3) / 65536: an
//   integer-exact approximation of N(0, sigma^2) (range +-3.46 sigma), so the
//   host and the device produce identical bits without transcendentals.
#pragma once

#include <stdint.h>

namespace n550 {

__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__host__ __device__ __forceinline__ uint64_t synth_key(uint64_t seed, uint64_t stream) {
    return splitmix64(seed ^ splitmix64(stream));
}

__host__ __device__ __forceinline__ uint64_t synth_u64(uint64_t key, uint64_t i) {
    return splitmix64(key + i * 0xD1B54A32D192ED03ull);
}

inline float synth_normal_scale(double sigma) {
    return (float)(sigma * 1.7320508075688772 / 65536.0);
}

__host__ __device__ __forceinline__ float synth_normal(uint64_t r, float scale) {
    const int s = (int)(r & 0xFFFF) + (int)((r >> 16) & 0xFFFF) + (int)((r >> 32) & 0xFFFF) +
                  (int)(r >> 48);
#ifdef __CUDA_ARCH__
    return __fmul_rn((float)(s - 131070), scale);
#else
    return (float)(s - 131070) * scale;
#endif
}

}  // namespace n550
