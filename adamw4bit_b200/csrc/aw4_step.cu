// aw4_step.cu -- the fused 4-bit AdamW step (one launch over many tensors).
//
// Work unit: a tile of 64 quantization blocks (8192 values) of one tensor.
// A persistent grid of 256-thread CTAs walks the tiles of every tensor in the
// launch; each warp takes a strip of 8 blocks, two at a time: each 16-lane
// group owns one 128-value block and each lane 8 consecutive values, so a
// block is decoded, updated and re-encoded entirely in registers (block
// absmax by a warp reduction, EDEN sums through shared memory) with exactly
// one read and one write of every byte of state:
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
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "aw4_encode.cuh"
#include "aw4_host.h"

namespace aw4 {

constexpr int kMaxTensors = 300;   // tensors per launch (kernel parameter space)
constexpr int kMaxHypers = 8;      // distinct per-step scalar sets per FP32-state launch
// A tile is 64 blocks (8192 values) of one tensor.  Warp w takes its 8
// consecutive blocks 8w .. 8w+7 as 4 sub-blocks of 2 (one per 16-lane group)
// and writes its 8 new scales per moment (32 bytes) itself, so warps never
// wait for one another.  Measured on the full kernel (2^27 values), this is
// 5 % faster than collecting the tile's 64 scales per moment for 256-byte
// stores behind a CTA barrier, although the kernel's load/store skeleton
// alone reaches 99 % of the copy bandwidth with the 256-byte stores and 85 %
// with per-warp 32-byte ones: the full kernel is bound by instruction issue,
// and the barrier made its warps wait in step.
constexpr int kSubBlocks = 4;
constexpr int kStepBlocksPerTile = kSubBlocks * kBlocksPerTile;   // 64 blocks

struct KDesc {
    void* param;
    const void* grad;
    uint8_t* c1;
    float* s1;
    uint8_t* c2;
    float* s2;
    const float* d1;
    const float* d2;
    void* pc;            // BF16 model copy of the updated params, or null
    int64_t elem_offset;
    int32_t nblocks;
    int32_t tile_begin;
    uint32_t ordinal;
    int32_t flags;          // kPcMulticast
};
constexpr int32_t kPcMulticast = 1;     // pc is an NVLink multicast address (multimem stores)

// One hyper-parameter set as the kernel reads it: the caller's aw4_hyper plus
// host-derived constants of the fast denominator/update path (fast_bounds).
struct HyperDev {
    float w1, w2, decay, neg_step;
    float sqrt_bc2, eps, sr_bias, rcp_sqrt_bc2;   // rcp: RN(1 / sqrt_bc2)
    float sr_rbias;                               // RN(1 / sr_bias), 0: fast update SR off
    float pos_step;                               // lr / bc1 = -neg_step
    float bsc, rbsc;                              // sqrt_bc2 * 2^24 and RN(1 / bsc)
    float m1_fast_max, m2_fast_max;               // lane bounds of the fast path (-1: off)
    uint32_t step;
    PhiloxKey m1_key, m2_key;                     // key schedules of the SR streams
    float grad_scale;                             // multiplies multicast-reduced gradients
};

// One launch covers tensors of one hyper-parameter set, so every scalar is
// read from the parameter bank at a fixed offset (an instruction operand, no
// load); the host issues one launch per distinct set.
struct StepLaunch {
    aw4_scheme m1, m2;
    HyperDev h;
    int32_t n_tensors, n_tiles, eden;
    float one;                        // 1.0, read at run time (packed additions)
    KDesc t[kMaxTensors];
};
static_assert(sizeof(StepLaunch) <= 32000, "kernel parameter space");

struct StepSmem {
    SmemScheme s1, s2;
    float scratch[kThreads / 32][kWarpScratch];
    float scales[2][kStepBlocksPerTile];   // the tile's new m1 / m2 scales
};
// 8-byte table entries (s2), and float4 columns in each warp's EDEN scratch
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

// The update q[i] = RN(RN(neg_step * m1[i]) / den[i]) with
// den = RN(RN(RN(sqrt(m2)) / sqrt_bc2) + eps) (adamw.py:685, 743), for a lane
// whose values pass the fast-path bounds:
//  * sqrt: sqrt_nr on m2 * 2^48 (exact scaling; every nonzero m2 >= 2^-149
//    lands at or above 2^-101, where sqrt_nr is exact), carried negated;
//    m2 == 0 reads 2^-126, whose root vanishes against eps (fast_bounds);
//  * / sqrt_bc2: Markstein against bsc = sqrt_bc2 * 2^24, which undoes the
//    2^24 of the scaled root exactly;
//  * / den: Markstein with ny = rcp_nr(-den) = RN(-1/den) and the positive
//    numerator nt = pos_step * m1 = -t: q0 = nt*ny, r = nt + q0*den (exact),
//    q = q0 + r*ny.  Written this way a zero numerator of either sign yields
//    the IEEE zero of t/den.
__device__ __forceinline__ void update_fast(float q[8], const float m1[8], const float m2[8],
                                            const HyperDev& H, float one) {
    const f2 k48 = pk2(-0x1p48f, -0x1p48f), kmin = pk2(-0x1p-126f, -0x1p-126f);
    const f2 half = pk2(0.5f, 0.5f), nbsc = pk2(-H.bsc, -H.bsc), rb = pk2(H.rbsc, H.rbsc);
    const f2 neg1 = pk2(-one, -one), eps = pk2(H.eps, H.eps), one2 = pk2(one, one);
    const f2 ps = pk2(H.pos_step, H.pos_step);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        // N = -(m2 * 2^48 + 2^-126): the sum rounds back to m2 * 2^48 unless m2 == 0
        const f2 N = f2_fma(pk2(m2[i], m2[i + 1]), k48, kmin);
        float n0, n1;
        upk2(N, n0, n1);
        const f2 y = pk2(rsqrt_approx(-n0), rsqrt_approx(-n1));
        const f2 ns = f2_mul(N, y);                        // -s
        const f2 h = f2_mul(half, y);
        const f2 nr = f2_fma(ns, ns, N);                   // s^2 - x = -r
        const f2 nroot = f2_fma(nr, h, ns);                // -(s + r*h) = -RN(sqrt(x))
        // nd = -RN(root / bsc)
        const f2 q0 = f2_mul(nroot, rb);
        const f2 r0 = f2_fma(q0, nbsc, nroot);
        const f2 nd = f2_fma(r0, rb, q0);
        const f2 den = f2_fma(nd, neg1, eps);              // RN(d + eps)
        float d0, d1;
        upk2(den, d0, d1);
        const f2 y0 = pk2(rcp_approx(-d0), rcp_approx(-d1));
        const f2 e = f2_fma(den, y0, one2);                // 1 - (-den) * y0
        const f2 ny = f2_fma(e, y0, y0);                   // RN(-1 / den)
        const f2 nt = f2_mul(pk2(m1[i], m1[i + 1]), ps);
        const f2 qa = f2_mul(nt, ny);
        const f2 rr = f2_fma(qa, den, nt);
        upk2(f2_fma(rr, ny, qa), q[i], q[i + 1]);
    }
}

// The same quantities by the IEEE operations, for lanes outside the bounds.
__device__ __forceinline__ void update_ieee(float q[8], const float m1[8], const float m2[8],
                                            const HyperDev& H) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float den = fadd(fdiv(fsqrt(m2[i]), H.sqrt_bc2), H.eps);
        q[i] = fdiv(fmul(H.neg_step, m1[i]), den);
    }
}

// The BF16 model copy of 8 updated values: a plain store, or, for a ZeRO-1
// model in symmetric memory, one multimem store to the NVLink multicast
// address, which NVSwitch delivers to every rank's replica.
__device__ __forceinline__ void store_model_copy(const KDesc& D, int64_t e0, const float p[8]) {
    if (!(D.flags & kPcMulticast)) {
        Elem<AW4_BF16>::store8(D.pc, e0, p);
        return;
    }
    const uint32_t w0 = pack_bf16x2(p[0], p[1]), w1 = pack_bf16x2(p[2], p[3]);
    const uint32_t w2 = pack_bf16x2(p[4], p[5]), w3 = pack_bf16x2(p[6], p[7]);
    uint16_t* dst = static_cast<uint16_t*>(D.pc) + e0;
    asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst),
                 "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                 : "memory");
}

// SR uniforms of 8 values: the test-hook draws buffer when given, else the
// in-kernel Philox stream of the moment.  For the update-SR rule (MODE
// AW4_SR_UPDATE) they are scaled by 2^24 (exact), the form its encoder takes.
template <int MODE>
__device__ __forceinline__ void load_uniforms(float u[8], const float* draws,
                                              const PhiloxKey& key, const HyperDev& H,
                                              const KDesc& D, int64_t e0, bool active) {
    constexpr bool scaled = MODE == AW4_SR_UPDATE;
    if (draws != nullptr && active) {
        Elem<AW4_F32>::load8(draws, e0, u);
        if (scaled) vmuls8(u, u, 0x1p24f);
    } else {
        philox_uniform8<scaled>(key, H.step, D.ordinal, (uint64_t)(D.elem_offset + e0), u);
    }
}

// GMC: the launch's gradients are multicast addresses (ZeRO-2), read as the
// sum over ranks; a separate instantiation keeps the plain load branch-free.
template <int PT, int GT, int M1, int M2, bool GMC>
__global__ void __launch_bounds__(kThreads, 4)
step_kernel(const __grid_constant__ StepLaunch L) {
    // F1: m1 is kept as float32 values (c1 holds them; no codes, no scales)
    constexpr bool F1 = M1 == AW4_FP32_MOMENT;
    __shared__ __align__(16) StepSmem sm;
    const int tid = threadIdx.x;
    if (!F1) load_scheme(sm.s1, L.m1, tid, kThreads);
    load_scheme(sm.s2, L.m2, tid, kThreads);
    __syncthreads();

    const int lane = tid & 31;
    const float one = L.one;
    const GroupCtx g = group_ctx(sm.scratch[tid >> 5], lane, one);
    const SchemeRegs r1 = scheme_regs(sm.s1, lane), r2 = scheme_regs(sm.s2, lane);
    const int warp = tid >> 5;
    const int h = lane >> 4;   // group within the warp
    const int zf2 = L.m2.zero_floor;

    // tiles only grow along this loop, so the owning tensor moves forward
    int ti = find_tensor(L, blockIdx.x);
    for (int tile = blockIdx.x; tile < L.n_tiles; tile += gridDim.x) {
        while (ti + 1 < L.n_tensors && L.t[ti + 1].tile_begin <= tile) ++ti;
        const KDesc& D = L.t[ti];
        const HyperDev& H = L.h;
        const int tile0 = (tile - D.tile_begin) * kStepBlocksPerTile;
        // ZeRO-2: each sub-block's gradient sums are requested from the
        // switch one sub-block ahead, so their round trip overlaps the math
        uint32_t gnext[8] = {0, 0, 0, 0, 0, 0, 0, 0};   // stays 0 past the tensor end
        if constexpr (GMC) {
            const int blk = tile0 + 8 * warp + h;
            if (blk < D.nblocks) issue8_reduce<GT>(D.grad, (int64_t)blk * kBlock + 8 * g.j, gnext);
        }
#pragma unroll 1
        for (int sb = 0; sb < kSubBlocks; ++sb) {
            const int slot = 8 * warp + 2 * sb + h;   // block within the tile: 8 per warp
            const int blk = tile0 + slot;
            const bool active = blk < D.nblocks;
            const int64_t e0 = (int64_t)blk * kBlock + 8 * g.j;
            uint32_t gcur[8];
            if constexpr (GMC) {
#pragma unroll
                for (int k = 0; k < 8; ++k) gcur[k] = gnext[k];
                if (sb + 1 < kSubBlocks && blk + 2 < D.nblocks)
                    issue8_reduce<GT>(D.grad, e0 + 2 * kBlock, gnext);
            }

            float p[8], gr[8], m1[8], m2[8];
            uint32_t w1 = 0, w2 = 0;
            float s1 = 0.0f, s2 = 0.0f;
            {
                // an inactive group reads the tensor's last block (never stored)
                const int blk = min(tile0 + slot, D.nblocks - 1);
                const int64_t e0 = (int64_t)blk * kBlock + 8 * g.j;
                Elem<PT>::load8(D.param, e0, p);
                if constexpr (GMC) {   // grad is a multicast address: the sum over ranks
                    finish8_reduce<GT>(gcur, gr);
                    vmuls8(gr, gr, H.grad_scale);
                } else {
                    Elem<GT>::load8(D.grad, e0, gr);
                }
                if constexpr (F1) {
                    Elem<AW4_F32>::load8(D.c1, e0, m1);
                    w2 = __ldcs(reinterpret_cast<const unsigned int*>(D.c2 + (e0 >> 1)));
                    s2 = __ldcs(D.s2 + blk);
                } else {
                    w1 = __ldcs(reinterpret_cast<const unsigned int*>(D.c1 + (e0 >> 1)));
                    w2 = __ldcs(reinterpret_cast<const unsigned int*>(D.c2 + (e0 >> 1)));
                    s1 = __ldcs(D.s1 + blk);
                    s2 = __ldcs(D.s2 + blk);
                }
            }
            // Packed f32x2 arithmetic throughout: multiplies, FMAs, and
            // additions as fma(a, one, b) (no multiply can be fused into them).
            // decode (quantization.py:996-999)
            float d[8], q[8];
            if (!F1) decode8s(fmul(r1.cbv, s1), w1, m1);
            decode8s(fmul(r2.cbv, s2), w2, m2);
            vfmas8(d, -one, m1, gr);                 // g - m1
            vfmas8(m1, H.w1, d, m1);                 // m1.lerp_(g, 1-b1)  (adamw.py:557)
            vmul8(q, gr, gr);                        // g*g
            vfmas8(d, -one, m2, q);                  // g*g - m2
            vfmas8(m2, H.w2, d, m2);                 // m2.lerp_(g*g, 1-b2) (adamw.py:684)
            const float amax1 = lane_absmax(m1), amax2 = lane_absmax(m2);
            float nt[8];
            vmuls8(nt, m1, H.pos_step);

            // One warp-uniform decision per sub-block: when every lane meets the
            // fast preconditions the rest runs without per-lane branches.  The
            // smallest magnitude among the values later divided (nt, and m1 or
            // m2 where SR or EDEN divides them) settles the tiny-value
            // precondition with one compare and one vote; only when some lane
            // holds a zero or a value below 2^-100 do the exact per-value tests
            // run, and the warp votes again on their result.
            // (an FP32 m1 has no block scale: 0 passes the divisor bound below)
            const float sc1 = F1 ? 0.0f : max_nan(group_max16(amax1), kScaleFloor);
            const float gmax2 = group_max16(amax2);
            const float sc2 = max_nan(gmax2, kScaleFloor);
            const bool lane_ok = active && amax1 <= H.m1_fast_max && amax2 <= H.m2_fast_max &&
                      sc1 <= kMarksteinMaxDivisor && sc2 <= kMarksteinMaxDivisor &&
                      (gmax2 >= kScaleFloor || !L.eden);
            const bool chk2 = M2 != AW4_RTN || L.eden;
            float mn = lane_absmin(nt);
            if (M1 == AW4_SR_VALUE) mn = fminf(mn, lane_absmin(m1));
            if (chk2) mn = fminf(mn, lane_absmin(m2));
            bool all = __all_sync(0xffffffffu, lane_ok && mn >= kMarksteinMinNumerator);
            if (!all) {   // a zero or a tiny value somewhere: the exact per-value tests
                bool ok = lane_ok && !any_tiny(nt);
                if (M1 == AW4_SR_VALUE) ok = ok && !any_tiny(m1);
                if (chk2) ok = ok && !any_tiny(m2);
                all = __all_sync(0xffffffffu, ok);
            }
            float u[8];
            if (all) {
                update_fast(q, m1, m2, H, one);
                vmuls8(p, p, H.decay);               // p.mul_(1 - lr*wd)
#pragma unroll
                for (int i = 0; i < 8; ++i) p[i] = Elem<PT>::round(p[i]);
                vadd8(p, q, p, one);                 // p.addcdiv_(m1, den, -lr/bc1)
                Elem<PT>::store8(D.param, e0, p);
                if (D.pc != nullptr) store_model_copy(D, e0, p);
                if constexpr (F1) {
                    Elem<AW4_F32>::store8(D.c1, e0, m1);   // the FP32 moment itself
                    if (M2 != AW4_RTN) load_uniforms<M2>(u, D.d2, H.m2_key, H, D, e0, true);
                    float ns2;
                    const uint32_t c2 =
                        encode_fast<M2>(sm.s2, r2, g, m2, sc2, u, zf2, L.eden, H.sr_bias, H.eps,
                                        H.sr_rbias, one, &ns2);
                    __stcs(reinterpret_cast<unsigned int*>(D.c2 + (e0 >> 1)), c2);
                    sm.scales[1][slot] = ns2;   // the same value from every lane of the group
                } else {
                    if (M1 == AW4_SR_VALUE) load_uniforms<M1>(u, D.d1, H.m1_key, H, D, e0, true);
                    float ns1, ns2;
                    const uint32_t c1 =
                        encode_fast<M1>(sm.s1, r1, g, m1, sc1, u, 0, 0, H.sr_bias, H.eps,
                                        H.sr_rbias, one, &ns1);
                    if (M2 != AW4_RTN) load_uniforms<M2>(u, D.d2, H.m2_key, H, D, e0, true);
                    const uint32_t c2 =
                        encode_fast<M2>(sm.s2, r2, g, m2, sc2, u, zf2, L.eden, H.sr_bias, H.eps,
                                        H.sr_rbias, one, &ns2);
                    __stcs(reinterpret_cast<unsigned int*>(D.c1 + (e0 >> 1)), c1);
                    __stcs(reinterpret_cast<unsigned int*>(D.c2 + (e0 >> 1)), c2);
                    sm.scales[0][slot] = ns1;   // the same value from every lane of the group
                    sm.scales[1][slot] = ns2;
                }
                continue;
            }

            // general path: per-lane guards, IEEE fallbacks, inactive groups
            if (amax1 <= H.m1_fast_max && amax2 <= H.m2_fast_max && !any_tiny(nt)) {
                update_fast(q, m1, m2, H, one);
            } else {
                update_ieee(q, m1, m2, H);
            }
            vmuls8(p, p, H.decay);                   // p.mul_(1 - lr*wd)
#pragma unroll
            for (int i = 0; i < 8; ++i) p[i] = Elem<PT>::round(p[i]);
            vadd8(p, q, p, one);                     // p.addcdiv_(m1, den, -lr/bc1)
            if (active) {
                Elem<PT>::store8(D.param, e0, p);
                if (D.pc != nullptr) store_model_copy(D, e0, p);
            }

            // re-encode m2 (adamw.py:675-683 update-SR, 795-803 RTN + floor + EDEN)
            // after m1 (adamw.py:764-771), or next to the FP32 moment itself
            if constexpr (F1) {
                if (active) Elem<AW4_F32>::store8(D.c1, e0, m1);
                if (M2 != AW4_RTN) load_uniforms<M2>(u, D.d2, H.m2_key, H, D, e0, active);
                float ns2;
                const uint32_t c2 = encode_block<M2>(sm.s2, r2, g, m2, amax2, u, zf2, L.eden,
                                                     H.sr_bias, H.eps, &ns2);
                if (active) {
                    __stcs(reinterpret_cast<unsigned int*>(D.c2 + (e0 >> 1)), c2);
                    if (g.j == 0) sm.scales[1][slot] = ns2;
                }
            } else {
                if (M1 == AW4_SR_VALUE) load_uniforms<M1>(u, D.d1, H.m1_key, H, D, e0, active);
                float ns1;
                const uint32_t c1 =
                    encode_block<M1>(sm.s1, r1, g, m1, amax1, u, 0, 0, H.sr_bias, H.eps, &ns1);
                if (M2 != AW4_RTN) load_uniforms<M2>(u, D.d2, H.m2_key, H, D, e0, active);
                float ns2;
                const uint32_t c2 = encode_block<M2>(sm.s2, r2, g, m2, amax2, u, zf2, L.eden,
                                                     H.sr_bias, H.eps, &ns2);
                if (active) {
                    __stcs(reinterpret_cast<unsigned int*>(D.c1 + (e0 >> 1)), c1);
                    __stcs(reinterpret_cast<unsigned int*>(D.c2 + (e0 >> 1)), c2);
                    if (g.j == 0) {
                        sm.scales[0][slot] = ns1;
                        sm.scales[1][slot] = ns2;
                    }
                }
            }
        }
        // this warp's 8 scales per moment: lanes 0-7 m1, 8-15 m2
        __syncwarp();
        if (lane < 16 && (!F1 || lane >= 8)) {
            const int k = lane & 7, mo = lane >> 3;
            const int tb = tile0 + 8 * warp + k;
            if (tb < D.nblocks) __stcs((mo ? D.s2 : D.s1) + tb, sm.scales[mo][8 * warp + k]);
        }
        __syncwarp();
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

template <int PT, int GT, int M1, bool GMC>
static StepFn pick_m2(int m2) {
    switch (m2) {
    case AW4_RTN: return step_kernel<PT, GT, M1, AW4_RTN, GMC>;
    case AW4_SR_VALUE: return step_kernel<PT, GT, M1, AW4_SR_VALUE, GMC>;
    case AW4_SR_UPDATE: return step_kernel<PT, GT, M1, AW4_SR_UPDATE, GMC>;
    }
    return nullptr;
}

template <int PT, int GT, bool GMC>
static StepFn pick_m1(int m1, int m2) {
    if (m1 == AW4_RTN) return pick_m2<PT, GT, AW4_RTN, GMC>(m2);
    if (m1 == AW4_SR_VALUE) return pick_m2<PT, GT, AW4_SR_VALUE, GMC>(m2);
    if constexpr (!GMC) {   // FP32 first moments next to a 4-bit second moment
        if (m1 == AW4_FP32_MOMENT) return pick_m2<PT, GT, AW4_FP32_MOMENT, false>(m2);
    }
    return nullptr;
}

template <bool GMC>
static StepFn pick_dtypes(int pdt, int gdt, int m1, int m2) {
    if (pdt == AW4_F32 && gdt == AW4_F32) return pick_m1<AW4_F32, AW4_F32, GMC>(m1, m2);
    if (pdt == AW4_F32 && gdt == AW4_BF16) return pick_m1<AW4_F32, AW4_BF16, GMC>(m1, m2);
    if (pdt == AW4_F32 && gdt == AW4_F16) return pick_m1<AW4_F32, AW4_F16, GMC>(m1, m2);
    if (pdt == AW4_BF16 && gdt == AW4_BF16) return pick_m1<AW4_BF16, AW4_BF16, GMC>(m1, m2);
    if (pdt == AW4_F16 && gdt == AW4_F16) return pick_m1<AW4_F16, AW4_F16, GMC>(m1, m2);
    return nullptr;
}

// Supported (param, grad) dtype pairs: equal dtypes, or FP32 master params
// with BF16/FP16 gradients; gmc selects the multicast-reduced gradient read.
static StepFn pick_step(int pdt, int gdt, int m1, int m2, bool gmc) {
    return gmc ? pick_dtypes<true>(pdt, gdt, m1, m2) : pick_dtypes<false>(pdt, gdt, m1, m2);
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

// A hyper-parameter set with the constants and lane bounds of update_fast.
// The fast path needs (every bound below is checked per lane in the kernel):
//  * eps in [2^-100, 2^25]: den = d + eps is normal and, with d <= 2^24, at
//    most 2^26 (Markstein's divisor range);
//  * sqrt_bc2 in [2^-76, 1]: bsc = sqrt_bc2 * 2^24 lies in Markstein's
//    divisor range;
//  * m2 in [0, 2^48 * bc2]: the scaled root stays finite and d <= 2^24; m2 is
//    non-negative when the m2 codebook is and 0 <= w2 <= 1 (the lerp is then a
//    convex combination under rounding);
//  * m2 == 0 reads 2^-126 in the scaled domain, so d = RN(2^-87 / sqrt_bc2)
//    instead of 0; that must stay below half an ulp of eps, so den == eps
//    exactly as with d == 0;
//  * |m1| <= 2^120 * min(eps, 1) / pos_step: nt and the quotient stay finite;
//  * every nt is zero or of magnitude >= 2^-100 (checked in the kernel).
static HyperDev hyper_dev(const aw4_hyper& h, const aw4_scheme& m2s) {
    HyperDev d;
    std::memset(&d, 0, sizeof(d));
    d.w1 = h.w1;
    d.w2 = h.w2;
    d.decay = h.decay;
    d.neg_step = h.neg_step;
    d.sqrt_bc2 = h.sqrt_bc2;
    d.eps = h.eps;
    d.sr_bias = h.sr_bias;
    d.sr_rbias = sr_fast_rbias(h.sr_bias, h.eps);
    d.step = h.step;
    d.m1_key = philox_schedule(h.m1_key);
    d.m2_key = philox_schedule(h.m2_key);
    d.grad_scale = h.grad_scale;
    d.pos_step = -h.neg_step;
    d.bsc = h.sqrt_bc2 * 0x1p24f;
    // float32 divisions on the host (SSE): correctly rounded
    volatile float one = 1.0f;
    d.rcp_sqrt_bc2 = one / h.sqrt_bc2;
    d.rbsc = one / d.bsc;
    d.m1_fast_max = -1.0f;   // off: no lane passes
    d.m2_fast_max = -1.0f;
    float cb_min = m2s.codebook[0];
    for (int k = 1; k < 16; ++k) cb_min = std::min(cb_min, m2s.codebook[k]);
    const double eps = h.eps, sb = h.sqrt_bc2, ps = d.pos_step;
    const bool ok = cb_min >= 0.0f && h.w2 >= 0.0f && h.w2 <= 1.0f && eps >= 0x1p-100 &&
                    eps <= 0x1p25 && sb >= 0x1p-76 && sb <= 1.0 && ps >= 0.0 &&
                    ps <= 3.0e38;
    if (!ok) return d;
    const double ulp_eps = (double)std::nextafter(h.eps, INFINITY) - eps;
    if (!(0x1p-87 / sb * (1.0 + 0x1p-20) < 0.5 * ulp_eps)) return d;
    d.m2_fast_max = (float)(0x1p48 * sb * sb * (1.0 - 0x1p-20));
    const double m1max = 0x1p120 * std::min(eps, 1.0) / std::max(ps, 1e-300);
    d.m1_fast_max = (float)std::min(m1max, 3.0e38);
    return d;
}

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
    if (m1->round_mode != AW4_RTN && m1->round_mode != AW4_SR_VALUE &&
        m1->round_mode != AW4_FP32_MOMENT)
        return fail(AW4_ERR_UNSUPPORTED,
                    "aw4_step_quantized: m1 must be RTN, value SR or an FP32 moment");
    const bool f1 = m1->round_mode == AW4_FP32_MOMENT;
    if (m2->round_mode < AW4_RTN || m2->round_mode > AW4_SR_UPDATE)
        return fail(AW4_ERR_INVALID, "aw4_step_quantized: bad m2 rounding mode");
    StepFn fn = pick_step(param_dtype, grad_dtype, m1->round_mode, m2->round_mode, false);
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
        if (!t.param || !t.grad || !t.m1_codes || (!t.m1_scales && !f1) || !t.m2_codes ||
            !t.m2_scales)
            return fail(AW4_ERR_INVALID, "tensor %d: null buffer", i);
        if (f1 && (!aligned(t.m1_codes, 16) || t.grad_multicast))
            return fail(AW4_ERR_INVALID, "tensor %d: an FP32 m1 needs 16-byte aligned values and "
                        "a local gradient", i);
        if (!aligned(t.param, 16) || !aligned(t.grad, 16) || !aligned(t.m1_codes, 4) ||
            !aligned(t.m2_codes, 4) || !aligned(t.m1_scales, 4) || !aligned(t.m2_scales, 4) ||
            (t.m1_draws && !aligned(t.m1_draws, 16)) || (t.m2_draws && !aligned(t.m2_draws, 16)))
            return fail(AW4_ERR_INVALID, "tensor %d: misaligned buffer (16 B for values, 4 B codes)",
                        i);
        if (t.elem_offset < 0 || t.elem_offset % AW4_BLOCK != 0)
            return fail(AW4_ERR_INVALID, "tensor %d: elem_offset must be a multiple of 128", i);
        if (t.hyper < 0 || t.hyper >= n_hypers)
            return fail(AW4_ERR_INVALID, "tensor %d: hyper index %d out of range", i, t.hyper);
        if (t.param_copy && (param_dtype != AW4_F32 || !aligned(t.param_copy, 16)))
            return fail(AW4_ERR_INVALID,
                        "tensor %d: a BF16 param copy needs FP32 params and 16-byte alignment", i);
        (void)pb; (void)gb;
    }
    DeviceGuard guard(device);
    if (!guard.ok()) return fail(AW4_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int grid_cap = grid_for(fn, device, 1 << 30);
    if (max_ctas > 0) grid_cap = std::min(grid_cap, max_ctas);

    // Distinct (hyper-parameter set, gradient kind) pairs (equal hyper
    // contents count as one), then one or more launches of <= kMaxTensors
    // tensors per pair.
    std::vector<int> set_of(n_tensors, -1), reps;
    for (int i = 0; i < n_tensors; ++i) {
        for (size_t k = 0; k < reps.size(); ++k)
            if ((tensors[reps[k]].grad_multicast != 0) == (tensors[i].grad_multicast != 0) &&
                (tensors[reps[k]].hyper == tensors[i].hyper ||
                 std::memcmp(&hypers[tensors[reps[k]].hyper], &hypers[tensors[i].hyper],
                             sizeof(aw4_hyper)) == 0)) {
                set_of[i] = (int)k;
                break;
            }
        if (set_of[i] < 0) {
            set_of[i] = (int)reps.size();
            reps.push_back(i);
        }
    }
    StepLaunch* L = new StepLaunch;
    std::memset(L, 0, sizeof(StepLaunch));
    L->m1 = *m1;
    L->m2 = *m2;
    L->eden = eden ? 1 : 0;
    L->one = 1.0f;
    int32_t rc = AW4_OK;
    for (size_t set = 0; set < reps.size() && rc == AW4_OK; ++set) {
        L->h = hyper_dev(hypers[tensors[reps[set]].hyper], *m2);
        // same resources as fn (launch bounds, shared memory): same grid cap
        const StepFn sfn = tensors[reps[set]].grad_multicast
                               ? pick_step(param_dtype, grad_dtype, m1->round_mode,
                                           m2->round_mode, true)
                               : fn;
        int i = 0;
        while (i < n_tensors && rc == AW4_OK) {
            L->n_tensors = 0;
            L->n_tiles = 0;
            for (; i < n_tensors && L->n_tensors < kMaxTensors; ++i) {
                const aw4_qtensor& t = tensors[i];
                if (t.numel == 0 || set_of[i] != (int)set) continue;
                KDesc& d = L->t[L->n_tensors++];
                d.param = t.param;
                d.grad = t.grad;
                d.c1 = t.m1_codes;
                d.s1 = t.m1_scales;
                d.c2 = t.m2_codes;
                d.s2 = t.m2_scales;
                d.d1 = t.m1_draws;
                d.d2 = t.m2_draws;
                d.pc = t.param_copy;
                d.flags = (t.param_copy && t.copy_multicast) ? kPcMulticast : 0;
                d.elem_offset = t.elem_offset;
                d.nblocks = (int32_t)(t.numel / AW4_BLOCK);
                d.tile_begin = L->n_tiles;
                d.ordinal = t.ordinal;
                const int64_t tiles = (d.nblocks + kStepBlocksPerTile - 1) / kStepBlocksPerTile;
                if ((int64_t)L->n_tiles + tiles > 0x7fffffffLL) {
                    rc = fail(AW4_ERR_INVALID, "launch exceeds 2^31 tiles");
                    break;
                }
                L->n_tiles += (int32_t)tiles;
            }
            if (rc != AW4_OK || L->n_tensors == 0) break;
            const int grid = std::min(grid_cap, L->n_tiles);
            sfn<<<grid, kThreads, 0, s>>>(*L);
            note_launch();
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) rc = fail(AW4_ERR_CUDA, "step launch: %s", cudaGetErrorString(e));
        }
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
