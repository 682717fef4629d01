// aw4_step.cu -- the fused 4-bit AdamW step (one launch over many tensors).
//
// Work unit: a tile of 16 quantization blocks (2048 values) of one tensor.
// A persistent grid of 256-thread CTAs walks the tiles of every tensor in the
// launch; each 16-lane group owns one 128-value block and each lane 8
// consecutive values, so a block is decoded, updated and re-encoded entirely
// in registers (block absmax by shuffles, EDEN sums through shared memory)
// with exactly one read and one write of every byte of state:
//   read  param, grad, m1/m2 packed codes, m1/m2 block scales
//   write param,       m1/m2 packed codes, m1/m2 block scales
//
// Reference semantics (nubank/adamw4bit, eager path, adamw.py:497-803):
//   m1 = cb1[c1] * s1,  m2 = cb2[c2] * s2            (quantization.py:975-1004)
//   m1 = fma(1-b1, g - m1, m1)                        (adamw.py:557, Tensor.lerp_)
//   m2 = fma(1-b2, g*g - m2, m2)                      (adamw.py:684)
//   den = sqrt(m2) / sqrt(bc2) + eps                  (adamw.py:685)
//   p = p * (1 - lr*wd); p = p + (-lr/bc1 * m1) / den  (adamw.py:691, 743)
//   store m1 (RTN, or value-SR after an nf4_sr switch) (adamw.py:764-771)
//   store m2 (RTN + zero floor + EDEN, or update-SR)  (adamw.py:675-683, 795-803)
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include "aw4_encode.cuh"
#include "aw4_host.h"

namespace aw4 {

constexpr int kMaxTensors = 300;   // tensors per launch (kernel parameter space)
constexpr int kMaxHypers = 8;      // distinct per-step scalar sets per launch

struct KDesc {
    void* param;
    const void* grad;
    uint8_t* c1;
    float* s1;
    uint8_t* c2;
    float* s2;
    const float* d1;
    const float* d2;
    int64_t elem_offset;
    int32_t nblocks;
    int32_t tile_begin;
    uint32_t ordinal;
    int32_t hyper;
};

struct StepLaunch {
    aw4_scheme m1, m2;
    aw4_hyper hyper[kMaxHypers];
    float rcp_sqrt_bc2[kMaxHypers];   // RN(1 / sqrt_bc2), IEEE division on the host
    int32_t n_tensors, n_tiles, eden, pad;
    KDesc t[kMaxTensors];
};
static_assert(sizeof(StepLaunch) <= 32000, "kernel parameter space");

struct StepSmem {
    SmemScheme s1, s2;
    float scratch[kThreads / 32][kWarpScratch];
};
// 16-byte table reads (s2), and float4 rows in each warp's EDEN scratch
static_assert(offsetof(StepSmem, s2) % 16 == 0, "");
static_assert(offsetof(StepSmem, scratch) % 16 == 0 && (kWarpScratch * 4) % 16 == 0, "");

__device__ __forceinline__ int find_tensor(const StepLaunch& L, int tile) {
    int lo = 0, hi = L.n_tensors - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.t[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <int PT, int GT, int M1, int M2>
__global__ void __launch_bounds__(kThreads, 4)
step_kernel(const __grid_constant__ StepLaunch L) {
    __shared__ __align__(16) StepSmem sm;
    const int tid = threadIdx.x;
    load_scheme(sm.s1, L.m1, tid, kThreads);
    load_scheme(sm.s2, L.m2, tid, kThreads);
    __syncthreads();

    const int lane = tid & 31;
    const GroupCtx g = group_ctx(sm.scratch[tid >> 5], lane);
    const SchemeRegs r1 = scheme_regs(sm.s1, lane), r2 = scheme_regs(sm.s2, lane);
    const int group = tid >> 4;
    const int zf2 = L.m2.zero_floor;

    // tiles only grow along this loop, so the owning tensor moves forward
    int ti = find_tensor(L, blockIdx.x);
    for (int tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x) {
        while (ti + 1 < L.n_tensors && L.t[ti + 1].tile_begin <= tile) ++ti;
        const KDesc& D = L.t[ti];
        const aw4_hyper& H = L.hyper[D.hyper];
        const int blk = (tile - D.tile_begin) * kBlocksPerTile + group;
        const bool active = blk < D.nblocks;
        const int64_t e0 = (int64_t)blk * kBlock + 8 * g.j;

        float p[8], gr[8], m1[8], m2[8];
        uint32_t w1 = 0, w2 = 0;
        float s1 = 0.0f, s2 = 0.0f;
        if (active) {
            Elem<PT>::load8(D.param, e0, p);
            Elem<GT>::load8(D.grad, e0, gr);
            w1 = __ldcs(reinterpret_cast<const unsigned int*>(D.c1 + (e0 >> 1)));
            w2 = __ldcs(reinterpret_cast<const unsigned int*>(D.c2 + (e0 >> 1)));
            s1 = __ldcs(D.s1 + blk);
            s2 = __ldcs(D.s2 + blk);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) p[i] = gr[i] = 0.0f;
        }
        // Packed f32x2 ops are used only where operand fusion cannot change a
        // result (FMA, and products consumed by an FMA, a division or a store):
        // ptxas may contract a packed mul.rn feeding a packed add/sub.rn into
        // one FMA, so every multiply -> add/sub chain below stays scalar.
        // decode (quantization.py:996-999)
        float d[8], t[8];
        decode8(r1.cbv, w1, s1, m1);
        decode8(r2.cbv, w2, s2, m2);
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = fsub(gr[i], m1[i]);
        vfmas8(m1, H.w1, d, m1);                 // m1.lerp_(g, 1-b1)  (adamw.py:557)
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = fsub(fmul(gr[i], gr[i]), m2[i]);
        vfmas8(m2, H.w2, d, m2);                 // m2.lerp_(g*g, 1-b2) (adamw.py:684)
        const float amax2 = lane_absmax(m2);
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = fsqrt(m2[i]);
        // den = sqrt(m2) / sqrt(bc2) + eps (adamw.py:685); sqrt of a finite
        // float is 0 or >= 2^-75, so Markstein's preconditions hold
        if (is_finite(amax2) && H.sqrt_bc2 >= kMarksteinMinDivisor &&
            H.sqrt_bc2 <= kMarksteinMaxDivisor) {
            vdiv_markstein8(d, t, H.sqrt_bc2, L.rcp_sqrt_bc2[D.hyper]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) d[i] = fdiv(t[i], H.sqrt_bc2);
        }
        vmuls8(t, m1, H.neg_step);               // (-lr/bc1) * m1, consumed by a division
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float den = fadd(d[i], H.eps);
            const float pd = Elem<PT>::round(fmul(p[i], H.decay));   // p.mul_(1 - lr*wd)
            p[i] = fadd(pd, fdiv(t[i], den));                       // p.addcdiv_(m1, den, -lr/bc1)
        }
        if (active) Elem<PT>::store8(D.param, e0, p);

        // re-encode m1 (adamw.py:764-771)
        float u[8];
        if (M1 != AW4_RTN) {
            if (D.d1 != nullptr && active) {
                const float4* q = reinterpret_cast<const float4*>(D.d1 + e0);
                const float4 a = __ldcs(q), b = __ldcs(q + 1);
                u[0] = a.x; u[1] = a.y; u[2] = a.z; u[3] = a.w;
                u[4] = b.x; u[5] = b.y; u[6] = b.z; u[7] = b.w;
            } else {
                philox_uniform8(H.m1_key, H.step, D.ordinal, (uint64_t)(D.elem_offset + e0), u);
            }
        }
        float ns1;
        const uint32_t c1 =
            encode_block<M1>(sm.s1, r1, g, m1, lane_absmax(m1), u, 0, 0, H.sr_bias, H.eps, &ns1);

        // re-encode m2 (adamw.py:675-683 update-SR, 795-803 RTN + floor + EDEN)
        if (M2 != AW4_RTN) {
            if (D.d2 != nullptr && active) {
                const float4* q = reinterpret_cast<const float4*>(D.d2 + e0);
                const float4 a = __ldcs(q), b = __ldcs(q + 1);
                u[0] = a.x; u[1] = a.y; u[2] = a.z; u[3] = a.w;
                u[4] = b.x; u[5] = b.y; u[6] = b.z; u[7] = b.w;
            } else {
                philox_uniform8(H.m2_key, H.step, D.ordinal, (uint64_t)(D.elem_offset + e0), u);
            }
        }
        float ns2;
        const uint32_t c2 =
            encode_block<M2>(sm.s2, r2, g, m2, amax2, u, zf2, L.eden, H.sr_bias, H.eps, &ns2);

        if (active) {
            __stcs(reinterpret_cast<unsigned int*>(D.c1 + (e0 >> 1)), c1);
            __stcs(reinterpret_cast<unsigned int*>(D.c2 + (e0 >> 1)), c2);
            if (g.j == 0) {
                __stcs(D.s1 + blk, ns1);
                __stcs(D.s2 + blk, ns2);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// FP32-state tensors (adamw.py:807-817 ineligible tensors: moments stay FP32)
// ---------------------------------------------------------------------------
constexpr int kMaxFTensors = 384;
constexpr int kFChunk = kThreads * 4;  // values per CTA iteration

struct FDesc {
    void* param;
    const void* grad;
    float* m1;
    float* m2;
    int64_t numel;
    int32_t chunk_begin;
    int32_t hyper;
};

struct FLaunch {
    aw4_hyper hyper[kMaxHypers];
    int32_t n_tensors, n_chunks;
    FDesc t[kMaxFTensors];
};
static_assert(sizeof(FLaunch) <= 32000, "kernel parameter space");

template <int PT, int GT>
__global__ void __launch_bounds__(kThreads) fp32_state_kernel(const __grid_constant__ FLaunch L) {
    for (int chunk = blockIdx.x; chunk < L.n_chunks; chunk += gridDim.x) {
        int lo = 0, hi = L.n_tensors - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (L.t[mid].chunk_begin <= chunk) lo = mid; else hi = mid - 1;
        }
        const FDesc& D = L.t[lo];
        const aw4_hyper& H = L.hyper[D.hyper];
        const int64_t base = (int64_t)(chunk - D.chunk_begin) * kFChunk;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t e = base + k * kThreads + threadIdx.x;
            if (e >= D.numel) break;
            const float gv = Elem<GT>::load1(D.grad, e);
            float m1 = D.m1[e], m2 = D.m2[e];
            m1 = ffma(H.w1, fsub(gv, m1), m1);
            m2 = ffma(H.w2, fsub(fmul(gv, gv), m2), m2);
            const float den = fadd(fdiv(fsqrt(m2), H.sqrt_bc2), H.eps);
            const float pd = Elem<PT>::round(fmul(Elem<PT>::load1(D.param, e), H.decay));
            Elem<PT>::store1(D.param, e, fadd(pd, fdiv(fmul(H.neg_step, m1), den)));
            D.m1[e] = m1;
            D.m2[e] = m2;
        }
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using StepFn = void (*)(StepLaunch);

template <int PT, int GT, int M1>
static StepFn pick_m2(int m2) {
    switch (m2) {
    case AW4_RTN: return step_kernel<PT, GT, M1, AW4_RTN>;
    case AW4_SR_VALUE: return step_kernel<PT, GT, M1, AW4_SR_VALUE>;
    case AW4_SR_UPDATE: return step_kernel<PT, GT, M1, AW4_SR_UPDATE>;
    }
    return nullptr;
}

template <int PT, int GT>
static StepFn pick_m1(int m1, int m2) {
    if (m1 == AW4_RTN) return pick_m2<PT, GT, AW4_RTN>(m2);
    if (m1 == AW4_SR_VALUE) return pick_m2<PT, GT, AW4_SR_VALUE>(m2);
    return nullptr;
}

// Supported (param, grad) dtype pairs: equal dtypes, or FP32 master params
// with BF16/FP16 gradients.
static StepFn pick_step(int pdt, int gdt, int m1, int m2) {
    if (pdt == AW4_F32 && gdt == AW4_F32) return pick_m1<AW4_F32, AW4_F32>(m1, m2);
    if (pdt == AW4_F32 && gdt == AW4_BF16) return pick_m1<AW4_F32, AW4_BF16>(m1, m2);
    if (pdt == AW4_F32 && gdt == AW4_F16) return pick_m1<AW4_F32, AW4_F16>(m1, m2);
    if (pdt == AW4_BF16 && gdt == AW4_BF16) return pick_m1<AW4_BF16, AW4_BF16>(m1, m2);
    if (pdt == AW4_F16 && gdt == AW4_F16) return pick_m1<AW4_F16, AW4_F16>(m1, m2);
    return nullptr;
}

using FFn = void (*)(FLaunch);

static FFn pick_fp32(int pdt, int gdt) {
    if (pdt == AW4_F32 && gdt == AW4_F32) return fp32_state_kernel<AW4_F32, AW4_F32>;
    if (pdt == AW4_F32 && gdt == AW4_BF16) return fp32_state_kernel<AW4_F32, AW4_BF16>;
    if (pdt == AW4_F32 && gdt == AW4_F16) return fp32_state_kernel<AW4_F32, AW4_F16>;
    if (pdt == AW4_BF16 && gdt == AW4_BF16) return fp32_state_kernel<AW4_BF16, AW4_BF16>;
    if (pdt == AW4_F16 && gdt == AW4_F16) return fp32_state_kernel<AW4_F16, AW4_F16>;
    return nullptr;
}

static int dtype_bytes(int dt) { return dt == AW4_F32 ? 4 : 2; }

static bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }

// Grid: a multiple of the SM count, at most the resident CTAs, at most the work.
template <typename Fn>
static int grid_for(Fn fn, int device, int work) {
    int sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads, 0);
    if (sms <= 0) sms = 1;
    if (per_sm <= 0) per_sm = 1;
    return std::max(1, std::min(work, sms * per_sm));
}

}  // namespace aw4

using namespace aw4;

extern "C" int32_t aw4_step_quantized(const aw4_scheme* m1, const aw4_scheme* m2, int32_t eden,
                                      int32_t param_dtype, int32_t grad_dtype,
                                      const aw4_qtensor* tensors, int32_t n_tensors,
                                      const aw4_hyper* hypers, int32_t n_hypers, int32_t max_ctas,
                                      int32_t device, void* stream) {
    if (!m1 || !m2 || (n_tensors > 0 && (!tensors || !hypers)) || n_tensors < 0 || n_hypers < 0)
        return fail(AW4_ERR_INVALID, "aw4_step_quantized: null argument or negative count");
    if (m1->round_mode != AW4_RTN && m1->round_mode != AW4_SR_VALUE)
        return fail(AW4_ERR_UNSUPPORTED, "aw4_step_quantized: m1 rounding must be RTN or value SR");
    if (m2->round_mode < AW4_RTN || m2->round_mode > AW4_SR_UPDATE)
        return fail(AW4_ERR_INVALID, "aw4_step_quantized: bad m2 rounding mode");
    StepFn fn = pick_step(param_dtype, grad_dtype, m1->round_mode, m2->round_mode);
    if (!fn)
        return fail(AW4_ERR_UNSUPPORTED,
                    "aw4_step_quantized: unsupported (param, grad) dtype pair %d/%d", param_dtype,
                    grad_dtype);
    const int pb = dtype_bytes(param_dtype), gb = dtype_bytes(grad_dtype);
    for (int i = 0; i < n_tensors; ++i) {
        const aw4_qtensor& t = tensors[i];
        if (t.numel < 0 || t.numel % AW4_BLOCK != 0 || t.numel / AW4_BLOCK > 0x7fffffffLL)
            return fail(AW4_ERR_INVALID, "tensor %d: numel %lld is not a positive multiple of 128",
                        i, (long long)t.numel);
        if (t.numel == 0) continue;
        if (!t.param || !t.grad || !t.m1_codes || !t.m1_scales || !t.m2_codes || !t.m2_scales)
            return fail(AW4_ERR_INVALID, "tensor %d: null buffer", i);
        if (!aligned(t.param, 16) || !aligned(t.grad, 16) || !aligned(t.m1_codes, 4) ||
            !aligned(t.m2_codes, 4) || !aligned(t.m1_scales, 4) || !aligned(t.m2_scales, 4) ||
            (t.m1_draws && !aligned(t.m1_draws, 16)) || (t.m2_draws && !aligned(t.m2_draws, 16)))
            return fail(AW4_ERR_INVALID, "tensor %d: misaligned buffer (16 B for values, 4 B codes)",
                        i);
        if (t.elem_offset < 0 || t.elem_offset % AW4_BLOCK != 0)
            return fail(AW4_ERR_INVALID, "tensor %d: elem_offset must be a multiple of 128", i);
        if (t.hyper < 0 || t.hyper >= n_hypers)
            return fail(AW4_ERR_INVALID, "tensor %d: hyper index %d out of range", i, t.hyper);
        (void)pb; (void)gb;
    }
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int grid_cap = grid_for(fn, device, 1 << 30);
    if (max_ctas > 0) grid_cap = std::min(grid_cap, max_ctas);

    // Pack tensors into launches of <= kMaxTensors tensors / kMaxHypers scalar sets.
    StepLaunch* L = new StepLaunch;
    std::memset(L, 0, sizeof(StepLaunch));
    L->m1 = *m1;
    L->m2 = *m2;
    L->eden = eden ? 1 : 0;
    int hmap[64];
    int i = 0;
    int32_t rc = AW4_OK;
    while (i < n_tensors && rc == AW4_OK) {
        L->n_tensors = 0;
        L->n_tiles = 0;
        int nh = 0;
        std::vector<int> hsrc;
        for (; i < n_tensors && L->n_tensors < kMaxTensors; ++i) {
            const aw4_qtensor& t = tensors[i];
            if (t.numel == 0) continue;
            int h = -1;
            for (int k = 0; k < nh; ++k)
                if (hsrc[k] == t.hyper ||
                    std::memcmp(&hypers[hsrc[k]], &hypers[t.hyper], sizeof(aw4_hyper)) == 0) {
                    h = k;
                    break;
                }
            if (h < 0) {
                if (nh == kMaxHypers) break;
                h = nh++;
                hsrc.push_back(t.hyper);
                L->hyper[h] = hypers[t.hyper];
                // IEEE float32 division (SSE on the host): correctly rounded
                volatile float one = 1.0f;
                L->rcp_sqrt_bc2[h] = one / hypers[t.hyper].sqrt_bc2;
            }
            (void)hmap;
            KDesc& d = L->t[L->n_tensors++];
            d.param = t.param;
            d.grad = t.grad;
            d.c1 = t.m1_codes;
            d.s1 = t.m1_scales;
            d.c2 = t.m2_codes;
            d.s2 = t.m2_scales;
            d.d1 = t.m1_draws;
            d.d2 = t.m2_draws;
            d.elem_offset = t.elem_offset;
            d.nblocks = (int32_t)(t.numel / AW4_BLOCK);
            d.tile_begin = L->n_tiles;
            d.ordinal = t.ordinal;
            d.hyper = h;
            const int64_t tiles = (d.nblocks + kBlocksPerTile - 1) / kBlocksPerTile;
            if ((int64_t)L->n_tiles + tiles > 0x7fffffffLL) {
                rc = fail(AW4_ERR_INVALID, "launch exceeds 2^31 tiles");
                break;
            }
            L->n_tiles += (int32_t)tiles;
        }
        if (rc != AW4_OK || L->n_tensors == 0) break;
        const int grid = std::min(grid_cap, L->n_tiles);
        fn<<<grid, kThreads, 0, s>>>(*L);
        note_launch();
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = fail(AW4_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
    }
    delete L;
    return rc;
}

extern "C" int32_t aw4_step_fp32_state(int32_t param_dtype, int32_t grad_dtype,
                                       const aw4_ftensor* tensors, int32_t n_tensors,
                                       const aw4_hyper* hypers, int32_t n_hypers, int32_t device,
                                       void* stream) {
    if ((n_tensors > 0 && (!tensors || !hypers)) || n_tensors < 0 || n_hypers < 0)
        return fail(AW4_ERR_INVALID, "aw4_step_fp32_state: null argument or negative count");
    FFn fn = pick_fp32(param_dtype, grad_dtype);
    if (!fn)
        return fail(AW4_ERR_UNSUPPORTED, "aw4_step_fp32_state: unsupported dtype pair %d/%d",
                    param_dtype, grad_dtype);
    for (int i = 0; i < n_tensors; ++i) {
        const aw4_ftensor& t = tensors[i];
        if (t.numel < 0) return fail(AW4_ERR_INVALID, "tensor %d: negative numel", i);
        if (t.numel == 0) continue;
        if (!t.param || !t.grad || !t.m1 || !t.m2)
            return fail(AW4_ERR_INVALID, "tensor %d: null buffer", i);
        if (t.hyper < 0 || t.hyper >= n_hypers)
            return fail(AW4_ERR_INVALID, "tensor %d: hyper index out of range", i);
    }
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid_cap = grid_for(fn, device, 1 << 30);
    FLaunch* L = new FLaunch;
    std::memset(L, 0, sizeof(FLaunch));
    int i = 0;
    int32_t rc = AW4_OK;
    while (i < n_tensors && rc == AW4_OK) {
        L->n_tensors = 0;
        L->n_chunks = 0;
        int nh = 0;
        std::vector<int> hsrc;
        for (; i < n_tensors && L->n_tensors < kMaxFTensors; ++i) {
            const aw4_ftensor& t = tensors[i];
            if (t.numel == 0) continue;
            int h = -1;
            for (int k = 0; k < nh; ++k)
                if (std::memcmp(&hypers[hsrc[k]], &hypers[t.hyper], sizeof(aw4_hyper)) == 0) {
                    h = k;
                    break;
                }
            if (h < 0) {
                if (nh == kMaxHypers) break;
                h = nh++;
                hsrc.push_back(t.hyper);
                L->hyper[h] = hypers[t.hyper];
            }
            FDesc& d = L->t[L->n_tensors++];
            d.param = t.param;
            d.grad = t.grad;
            d.m1 = t.m1;
            d.m2 = t.m2;
            d.numel = t.numel;
            d.chunk_begin = L->n_chunks;
            d.hyper = h;
            L->n_chunks += (int32_t)((t.numel + kFChunk - 1) / kFChunk);
        }
        if (L->n_tensors == 0) break;
        const int grid = std::min(grid_cap, L->n_chunks);
        fn<<<grid, kThreads, 0, s>>>(*L);
        note_launch();
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) rc = fail(AW4_ERR_CUDA, "fp32-state launch: %s", cudaGetErrorString(e));
    }
    delete L;
    return rc;
}
