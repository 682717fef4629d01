// aw4_selfcheck.cu -- exhaustive device check of rcp_nr and sqrt_nr.
//
// The step kernel's fast denominator/update path builds RN(1/b) and
// RN(sqrt(x)) from the hardware approximations (aw4_device.cuh).  This kernel
// compares both with the IEEE round-to-nearest operations on every float32 of
// the domains the step relies on:
//   rcp_nr(b)  for every b with 2^-126 <= |b| <= 2^126;
//   sqrt_nr(x) for every x in [2^-102, +inf) and x == 0 (the step feeds it
//   m2 * 2^48, which is 0 or at least 2^-101).
#include <cuda_runtime.h>

#include <algorithm>

#include "aw4_device.cuh"
#include "aw4_host.h"

namespace aw4 {

__global__ void __launch_bounds__(kThreads)
selfcheck_math_kernel(unsigned long long* counts) {
    unsigned long long bad_rcp = 0, bad_sqrt = 0;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (1ull << 32);
         i += stride) {
        const uint32_t bits = (uint32_t)i;
        const float x = __uint_as_float(bits);
        const float ax = fabsf(x);
        if (ax >= 0x1p-126f && ax <= 0x1p126f &&
            __float_as_uint(rcp_nr(x)) != __float_as_uint(__frcp_rn(x)))
            ++bad_rcp;
        if (((x >= 0x1p-102f && ax < __int_as_float(0x7f800000)) || bits == 0u) &&
            __float_as_uint(sqrt_nr(x)) != __float_as_uint(__fsqrt_rn(x)))
            ++bad_sqrt;
    }
    if (bad_rcp) atomicAdd(&counts[0], bad_rcp);
    if (bad_sqrt) atomicAdd(&counts[1], bad_sqrt);
}

}  // namespace aw4

using namespace aw4;

extern "C" int32_t aw4_selfcheck_math(uint64_t* counts, int32_t device, void* stream) {
    if (!counts) return fail(AW4_ERR_INVALID, "aw4_selfcheck_math: null counts");
    if (((uintptr_t)counts) % 8 != 0)
        return fail(AW4_ERR_INVALID, "aw4_selfcheck_math: counts must be 8-byte aligned");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(counts, 0, 2 * sizeof(uint64_t), s);
    if (e != cudaSuccess) return fail(AW4_ERR_CUDA, "aw4_selfcheck_math: %s", cudaGetErrorString(e));
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    selfcheck_math_kernel<<<std::max(sms, 1) * 8, kThreads, 0, s>>>(
        reinterpret_cast<unsigned long long*>(counts));
    note_launch();
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(AW4_ERR_CUDA, "aw4_selfcheck_math: %s", cudaGetErrorString(e));
    return AW4_OK;
}
