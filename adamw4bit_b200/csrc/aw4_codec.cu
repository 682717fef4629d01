// aw4_codec.cu -- standalone block codec, state initialisation and nibble
// packing (quantization.py:627-691, 715-1004; adamw.py:524-545).
#include <cuda_runtime.h>

#include <algorithm>

#include "aw4_encode.cuh"
#include "aw4_host.h"

namespace aw4 {

// Fills the packed codes and scales of an all-zero moment.
__global__ void __launch_bounds__(kThreads)
init_zero_kernel(uint8_t* codes, float* scales, int64_t n_code_words, int64_t n_blocks,
                 uint32_t code_word, float scale) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_code_words; i += stride)
        reinterpret_cast<uint32_t*>(codes)[i] = code_word;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_blocks; i += stride)
        scales[i] = scale;
}

// quantize(): one 16-lane group per 128-value block, persistent grid.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
quantize_kernel(const __grid_constant__ aw4_scheme scheme, int eden, const float* x,
                int64_t n_blocks, uint8_t* codes, float* scales, const float* draws,
                const PhiloxKey key, uint32_t step, uint32_t ordinal, float sr_bias,
                float sr_eps, float sr_rbias, float one) {
    __shared__ __align__(16) SmemScheme S;
    __shared__ __align__(16) float scratch[kThreads / 32][kWarpScratch];
    load_scheme(S, scheme, threadIdx.x, kThreads);
    __syncthreads();
    const GroupCtx g = group_ctx(scratch[threadIdx.x >> 5], threadIdx.x & 31, one);
    const SchemeRegs R = scheme_regs(S, threadIdx.x & 31);
    const int group = threadIdx.x >> 4;
    const int64_t n_tiles = (n_blocks + kBlocksPerTile - 1) / kBlocksPerTile;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int64_t blk = tile * kBlocksPerTile + group;
        const bool active = blk < n_blocks;
        const int64_t e0 = blk * kBlock + 8 * g.j;
        float v[8], u[8];
        if (active) {
            Elem<AW4_F32>::load8(x, e0, v);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = 0.0f;
        }
        if (MODE != AW4_RTN) {
            // update SR takes its draws scaled by 2^24 (exact)
            constexpr bool scaled = MODE == AW4_SR_UPDATE;
            if (draws != nullptr && active) {
                Elem<AW4_F32>::load8(draws, e0, u);
                if (scaled) vmuls8(u, u, 0x1p24f);
            } else {
                philox_uniform8<scaled>(key, step, ordinal, (uint64_t)e0, u);
            }
        }
        // the step kernel's dispatch: one warp vote selects the branch-free
        // encoder when every lane meets its preconditions (so the exhaustive
        // codec tests cover both encoders)
        float s;
        const float amax = lane_absmax(v);
        const float gmax = group_max16(amax);
        const float sc = max_nan(gmax, kScaleFloor);
        bool ok = sc <= kMarksteinMaxDivisor && (gmax >= kScaleFloor || !eden);   // false for NaN / inf
        if (MODE != AW4_RTN || eden) ok = none_tiny_warp(v, ok);
        // the fast update-SR encoder takes non-negative values (moments m2)
        if (MODE == AW4_SR_UPDATE) ok = ok && lane_min(v) >= 0.0f;
        const uint32_t c = __all_sync(0xffffffffu, ok)
                               ? encode_fast<MODE>(S, R, g, v, sc, u, scheme.zero_floor, eden,
                                                   sr_bias, sr_eps, sr_rbias, one, &s)
                               : encode_block<MODE>(S, R, g, v, amax, u, scheme.zero_floor, eden,
                                                    sr_bias, sr_eps, &s);
        if (active) {
            reinterpret_cast<uint32_t*>(codes)[e0 >> 3] = c;
            if (g.j == 0) scales[blk] = s;
        }
    }
}

__global__ void __launch_bounds__(kThreads)
dequantize_kernel(const __grid_constant__ aw4_scheme scheme, const uint8_t* codes,
                  const float* scales, int64_t n, float* out) {
    __shared__ float cb[16];
    if (threadIdx.x < 16) cb[threadIdx.x] = scheme.codebook[threadIdx.x];
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int code = (codes[i >> 1] >> ((i & 1) * 4)) & 15;
        out[i] = fmul(cb[code], scales[i / kBlock]);
    }
}

__global__ void __launch_bounds__(kThreads)
pack_kernel(const uint8_t* codes, int64_t n, uint8_t* packed) {
    const int64_t m = (n + 1) / 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < m; k += stride) {
        const uint8_t lo = codes[2 * k];
        const uint8_t hi = (2 * k + 1 < n) ? codes[2 * k + 1] : 0;
        packed[k] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
    }
}

__global__ void __launch_bounds__(kThreads)
unpack_kernel(const uint8_t* packed, int64_t n, uint8_t* codes) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        codes[i] = (packed[i >> 1] >> ((i & 1) * 4)) & 15;
}

// reduce_multicast(): out[8u .. 8u+7] = f32(sum over ranks) * scale, one
// 8-value unit per thread step.
template <int DT>
__global__ void __launch_bounds__(kThreads)
reduce_multicast_kernel(const void* mc, int64_t units, float scale, float* out) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += stride) {
        float v[8];
        load8_reduce<DT>(mc, 8 * u, v);
        vmuls8(v, v, scale);
        Elem<AW4_F32>::store8(out, 8 * u, v);
    }
}

static int grid_1d(int device, int64_t work_items) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (sms <= 0) sms = 1;
    const int64_t need = (work_items + kThreads - 1) / kThreads;
    return (int)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)sms * 8));
}

}  // namespace aw4

using namespace aw4;

extern "C" int32_t aw4_init_zero_state(const aw4_scheme* scheme, int32_t eden, uint8_t* codes,
                                       float* scales, int64_t numel, int32_t device,
                                       void* stream) {
    if (!scheme || numel < 0 || numel % AW4_BLOCK)
        return fail(AW4_ERR_INVALID, "aw4_init_zero_state: bad scheme or numel");
    if (numel == 0) return AW4_OK;
    if (!codes || !scales || ((uintptr_t)codes % 4) || ((uintptr_t)scales % 4))
        return fail(AW4_ERR_INVALID, "aw4_init_zero_state: null or misaligned buffer");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    const uint32_t byte = (uint32_t)scheme->zero_code | ((uint32_t)scheme->zero_code << 4);
    const uint32_t word = byte * 0x01010101u;
    const float sc = eden ? scheme->zero_scale_eden : scheme->zero_scale;
    const int64_t words = numel / 8, blocks = numel / AW4_BLOCK;
    init_zero_kernel<<<grid_1d(device, words), kThreads, 0, (cudaStream_t)stream>>>(
        codes, scales, words, blocks, word, sc);
    note_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AW4_OK : fail(AW4_ERR_CUDA, "init launch: %s", cudaGetErrorString(e));
}

extern "C" int32_t aw4_quantize_blocks(const aw4_scheme* scheme, int32_t eden, const float* x,
                                       int64_t numel, uint8_t* codes, float* scales,
                                       const float* draws, uint64_t key, uint32_t step,
                                       uint32_t ordinal, float sr_bias, float sr_eps,
                                       int32_t device, void* stream) {
    if (!scheme || numel < 0 || numel % AW4_BLOCK)
        return fail(AW4_ERR_INVALID, "aw4_quantize_blocks: numel must be a multiple of 128");
    if (numel == 0) return AW4_OK;
    if (!x || !codes || !scales || ((uintptr_t)x % 16) || ((uintptr_t)codes % 4) ||
        (draws && ((uintptr_t)draws % 16)))
        return fail(AW4_ERR_INVALID, "aw4_quantize_blocks: null or misaligned buffer");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    const int64_t n_blocks = numel / AW4_BLOCK;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    const int64_t tiles = (n_blocks + kBlocksPerTile - 1) / kBlocksPerTile;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, (int64_t)std::max(sms, 1) * 4));
    cudaStream_t s = (cudaStream_t)stream;
    const float rbias = sr_fast_rbias(sr_bias, sr_eps);
    const PhiloxKey pk = philox_schedule(key);
    switch (scheme->round_mode) {
    case AW4_RTN:
        quantize_kernel<AW4_RTN><<<grid, kThreads, 0, s>>>(*scheme, eden, x, n_blocks, codes, scales,
                                                           draws, pk, step, ordinal, sr_bias, sr_eps,
                                                           rbias, 1.0f);
        break;
    case AW4_SR_VALUE:
        quantize_kernel<AW4_SR_VALUE><<<grid, kThreads, 0, s>>>(*scheme, eden, x, n_blocks, codes,
                                                                scales, draws, pk, step, ordinal,
                                                                sr_bias, sr_eps, rbias, 1.0f);
        break;
    case AW4_SR_UPDATE:
        quantize_kernel<AW4_SR_UPDATE><<<grid, kThreads, 0, s>>>(*scheme, eden, x, n_blocks, codes,
                                                                 scales, draws, pk, step, ordinal,
                                                                 sr_bias, sr_eps, rbias, 1.0f);
        break;
    default:
        return fail(AW4_ERR_INVALID, "aw4_quantize_blocks: bad round mode");
    }
    note_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AW4_OK : fail(AW4_ERR_CUDA, "quantize launch: %s", cudaGetErrorString(e));
}

extern "C" int32_t aw4_dequantize_blocks(const aw4_scheme* scheme, const uint8_t* codes,
                                         const float* scales, int64_t numel, float* out,
                                         int32_t device, void* stream) {
    if (!scheme || numel < 0 || numel % AW4_BLOCK)
        return fail(AW4_ERR_INVALID, "aw4_dequantize_blocks: numel must be a multiple of 128");
    if (numel == 0) return AW4_OK;
    if (!codes || !scales || !out) return fail(AW4_ERR_INVALID, "aw4_dequantize_blocks: null buffer");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    dequantize_kernel<<<grid_1d(device, numel), kThreads, 0, (cudaStream_t)stream>>>(
        *scheme, codes, scales, numel, out);
    note_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AW4_OK : fail(AW4_ERR_CUDA, "dequantize launch: %s", cudaGetErrorString(e));
}

extern "C" int32_t aw4_pack_codes(const uint8_t* codes, int64_t numel, uint8_t* packed,
                                  int32_t device, void* stream) {
    if (numel < 0) return fail(AW4_ERR_INVALID, "aw4_pack_codes: negative numel");
    if (numel == 0) return AW4_OK;
    if (!codes || !packed) return fail(AW4_ERR_INVALID, "aw4_pack_codes: null buffer");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    pack_kernel<<<grid_1d(device, (numel + 1) / 2), kThreads, 0, (cudaStream_t)stream>>>(codes, numel,
                                                                                      packed);
    note_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AW4_OK : fail(AW4_ERR_CUDA, "pack launch: %s", cudaGetErrorString(e));
}

extern "C" int32_t aw4_unpack_codes(const uint8_t* packed, int64_t numel, uint8_t* codes,
                                    int32_t device, void* stream) {
    if (numel < 0) return fail(AW4_ERR_INVALID, "aw4_unpack_codes: negative numel");
    if (numel == 0) return AW4_OK;
    if (!codes || !packed) return fail(AW4_ERR_INVALID, "aw4_unpack_codes: null buffer");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    unpack_kernel<<<grid_1d(device, numel), kThreads, 0, (cudaStream_t)stream>>>(packed, numel, codes);
    note_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AW4_OK : fail(AW4_ERR_CUDA, "unpack launch: %s", cudaGetErrorString(e));
}

extern "C" int32_t aw4_reduce_multicast(const void* mc, int32_t dtype, int64_t numel, float scale,
                                        float* out, int32_t device, void* stream) {
    if (numel < 0 || numel % 8)
        return fail(AW4_ERR_INVALID, "aw4_reduce_multicast: numel must be a multiple of 8");
    if (numel == 0) return AW4_OK;
    if (!mc || !out || ((uintptr_t)mc % 16) || ((uintptr_t)out % 16))
        return fail(AW4_ERR_INVALID, "aw4_reduce_multicast: null or misaligned buffer");
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    const int64_t units = numel / 8;
    const int grid = grid_1d(device, units);
    cudaStream_t s = (cudaStream_t)stream;
    switch (dtype) {
    case AW4_F32:
        reduce_multicast_kernel<AW4_F32><<<grid, kThreads, 0, s>>>(mc, units, scale, out);
        break;
    case AW4_BF16:
        reduce_multicast_kernel<AW4_BF16><<<grid, kThreads, 0, s>>>(mc, units, scale, out);
        break;
    case AW4_F16:
        reduce_multicast_kernel<AW4_F16><<<grid, kThreads, 0, s>>>(mc, units, scale, out);
        break;
    default:
        return fail(AW4_ERR_INVALID, "aw4_reduce_multicast: bad dtype %d", dtype);
    }
    note_launch();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AW4_OK
                            : fail(AW4_ERR_CUDA, "reduce_multicast launch: %s", cudaGetErrorString(e));
}
