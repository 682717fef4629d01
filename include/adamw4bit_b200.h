/*
 * adamw4bit_b200.h -- C ABI of the B200-native fused 4-bit AdamW step.
 *
 * One shared library (adamw4bit_b200/libadamw4bit_b200.so, sm_100a) exports
 * these entry points.  They take plain device pointers, sizes, host-computed
 * float32 scalars and a CUDA stream handle (cudaStream_t passed as void*);
 * no torch types cross the boundary.  Every call is stream-ordered and
 * returns an aw4_status; on failure aw4_last_error() returns a message for
 * the calling thread.  The library never allocates or frees device memory:
 * every buffer belongs to the caller (the Python optimizer keeps them in its
 * state_dict-compatible per-parameter state).
 *
 * Reference interfaces replaced (nubank/adamw4bit, paths within the project):
 *   aw4_step_quantized      QuantizedAdamW.step, eligible-tensor branch
 *                           (src/adamw4bit/adamw.py:497-803) and the opt-in
 *                           chunked backend _step_parameter/_step_chunk
 *                           (src/adamw4bit/_optimized.py:145-234)
 *   aw4_step_fp32_state     QuantizedAdamW.step for TorchAO-ineligible tensors
 *                           (adamw.py:516-521, 807-817: FP32 moments)
 *   aw4_init_zero_state     state initialisation, _store of zero moments
 *                           (adamw.py:524-545; _moment_buffer.py:106-126)
 *   aw4_quantize_blocks     quantize / quantize_with_dequantized for 4-bit
 *                           schemes (src/adamw4bit/quantization.py:715-971)
 *   aw4_dequantize_blocks   dequantize (quantization.py:975-1004)
 *   aw4_pack_codes          pack_4bit_codes (quantization.py:627-638)
 *   aw4_unpack_codes        unpack_4bit_codes (quantization.py:641-654)
 *   aw4_scheme_prepare      codebook strategies (quantization.py:240-377,
 *                           401-552): turns a 16-level codebook into the
 *                           rounding tables the kernels use
 */
#ifndef ADAMW4BIT_B200_H
#define ADAMW4BIT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AW4_ABI_VERSION 5
#define AW4_BLOCK 128          /* elements per quantization block (4-bit default) */
#define AW4_LUT_BINS 1024      /* maximum uniform bins over [-1, 1] for the rounding search */

typedef enum aw4_status {
    AW4_OK = 0,
    AW4_ERR_INVALID = 1,       /* bad pointer, size, alignment or enum */
    AW4_ERR_CUDA = 2,          /* a CUDA runtime call failed */
    AW4_ERR_UNSUPPORTED = 3    /* valid request this build does not implement */
} aw4_status;

typedef enum aw4_dtype { AW4_F32 = 0, AW4_BF16 = 1, AW4_F16 = 2 } aw4_dtype;

/* How a moment's normalised values are rounded to one of 16 levels. */
typedef enum aw4_round {
    AW4_RTN = 0,         /* nearest level, ties up   (quantization.py:254-272) */
    AW4_SR_VALUE = 1,    /* value-unbiased SR        (quantization.py:286-315) */
    AW4_SR_UPDATE = 2,   /* preconditioner-space SR  (quantization.py:327-377) */
    AW4_FP32_MOMENT = 3  /* m1 only: kept as float32 values, not quantized (the "fp32"
                          * scheme next to a 4-bit m2, adamw.py:510-521, 830-833); the
                          * tensor's m1_codes points to numel float32 values (16-byte
                          * aligned) and m1_scales is unused */
} aw4_round;

/* A 4-bit moment scheme prepared for the kernels (host memory, filled by
 * aw4_scheme_prepare; the caller keeps it and passes it to every call). */
typedef struct aw4_scheme {
    float codebook[16];            /* sorted levels, bit-exact reference table */
    int32_t round_mode;            /* aw4_round */
    int32_t zero_floor;            /* 1: code 0 is stored as code 1 (dyn4_nz) */
    /* rounding search over lut_bins uniform bins of [-1, 1] (a power of two,
     * the fewest for which no bin holds two thresholds): x in bin
     * b = floor((x + 1) * lut_bins / 2) has code = lut[b] + (x >= thr[lut[b] + 1]);
     * lut[b] counts the thresholds at or below the bin's lower edge */
    int32_t lut_bins;
    uint8_t lut[AW4_LUT_BINS];
    float thr[18];                 /* thr[0] = -inf, thr[last] = +inf */
    float zero_scale;              /* block scale stored for an all-zero block */
    float zero_scale_eden;         /* ... and with EDEN calibration */
    uint8_t zero_code;             /* code stored for an all-zero block */
    uint8_t pad[3];
} aw4_scheme;

/* Per-step scalars of one parameter (or of a parameter group at one step),
 * derived in float64 exactly as the reference does and rounded to float32
 * where they meet float32 tensors (adamw.py:557-564, 684-691, 743):
 *   w1 = f32(1 - beta1)        w2 = f32(1 - beta2)
 *   decay = f32(1 - lr * wd)   neg_step = f32(-lr / (1 - beta1^t))
 *   sqrt_bc2 = f32(sqrt(1 - beta2^t))          eps = f32(eps)
 *   sr_bias = f32(max(storage bias correction, 1e-12))  (update SR only)
 * grad_scale multiplies gradients read through a multicast address
 * (aw4_qtensor.grad_multicast), e.g. 1/W to average over W ranks; other
 * gradients are used as given. */
typedef struct aw4_hyper {
    float w1, w2, decay, neg_step, sqrt_bc2, eps, sr_bias;
    uint32_t step;                 /* t, 1-based: Philox counter word */
    uint64_t m1_key, m2_key;       /* Philox keys of the m1 / m2 SR streams */
    float grad_scale;
    int32_t pad;                   /* zero */
} aw4_hyper;

/* One quantized tensor (or one contiguous shard of it, for ZeRO-1). */
typedef struct aw4_qtensor {
    void* param;                   /* numel values of the launch's param dtype */
    const void* grad;              /* numel values of the launch's grad dtype */
    uint8_t* m1_codes;             /* numel/2 bytes, even element in the low nibble */
    float* m1_scales;              /* numel/128 block scales */
    uint8_t* m2_codes;
    float* m2_scales;
    const float* m1_draws;         /* NULL: Philox; else numel uniforms in [0, 1) (test hook) */
    const float* m2_draws;
    int64_t numel;                 /* multiple of 128 */
    int64_t elem_offset;           /* index of element 0 in the whole tensor (Philox) */
    uint32_t ordinal;              /* parameter ordinal (Philox counter word) */
    int32_t hyper;                 /* index into the aw4_hyper array */
    void* param_copy;              /* NULL, or numel BF16 values that receive bf16(updated
                                    * param): the model copy of FP32 master parameters
                                    * (16-byte aligned; FP32 params only) */
    int32_t copy_multicast;        /* nonzero: param_copy is an NVLink multicast address
                                    * (an NVSwitch multicast object bound on every rank);
                                    * the copy is written with multimem stores and lands
                                    * in every rank's replica */
    int32_t grad_multicast;        /* nonzero: grad is an NVLink multicast address of a
                                    * gradient buffer bound on every rank; the kernel reads
                                    * the sum over ranks (multimem.ld_reduce: the switch
                                    * adds the ranks' values, BF16/F16 accumulated in FP32
                                    * (.acc::f32) and returned in the gradient dtype with
                                    * the switch's rounding, which on B200 is not
                                    * round-to-nearest-even) times the hyper
                                    * set's grad_scale (ZeRO-2: the gradient reduce-scatter
                                    * fused into the update) */
} aw4_qtensor;

/* One tensor with FP32 moments (numel arbitrary). */
typedef struct aw4_ftensor {
    void* param;
    const void* grad;
    float* m1;
    float* m2;
    int64_t numel;
    int32_t hyper;
    int32_t pad;
} aw4_ftensor;

/* Library identity and diagnostics. */
int32_t aw4_abi_version(void);
const char* aw4_last_error(void);
/* Number of kernels this library has launched so far (all devices). */
uint64_t aw4_launch_count(void);

/* Builds the rounding tables of a 16-level sorted codebook. */
int32_t aw4_scheme_prepare(const float* codebook16, int32_t round_mode, int32_t zero_floor,
                           aw4_scheme* out);

/* Fused AdamW step over quantized tensors: decode NF4/Dyn4 codes, AdamW in
 * FP32, parameter update, re-encode with block absmax scales (RTN or SR, the
 * optional dyn4_nz floor and EDEN on m2) and write packed codes back.  All
 * tensors of one call share the param/grad dtypes and the two schemes.
 * max_ctas > 0 caps the persistent grid (to leave SMs to a concurrent
 * collective); 0 fills the GPU. */
int32_t aw4_step_quantized(const aw4_scheme* m1, const aw4_scheme* m2, int32_t eden,
                           int32_t param_dtype, int32_t grad_dtype,
                           const aw4_qtensor* tensors, int32_t n_tensors,
                           const aw4_hyper* hypers, int32_t n_hypers, int32_t max_ctas,
                           int32_t device, void* stream);

/* AdamW step over tensors that keep FP32 moments. */
int32_t aw4_step_fp32_state(int32_t param_dtype, int32_t grad_dtype,
                            const aw4_ftensor* tensors, int32_t n_tensors,
                            const aw4_hyper* hypers, int32_t n_hypers,
                            int32_t device, void* stream);

/* Writes the packed codes and scales of an all-zero moment. */
int32_t aw4_init_zero_state(const aw4_scheme* scheme, int32_t eden, uint8_t* codes,
                            float* scales, int64_t numel, int32_t device, void* stream);

/* Standalone block codec (block 128): x[numel] float32 -> packed codes +
 * scales.  draws: NULL for Philox(key, step, ordinal) uniforms, else numel
 * uniforms in [0, 1).  bias/eps
 * are the update-SR bias correction (clamped at 1e-12) and Adam epsilon. */
int32_t aw4_quantize_blocks(const aw4_scheme* scheme, int32_t eden, const float* x,
                            int64_t numel, uint8_t* codes, float* scales,
                            const float* draws, uint64_t key, uint32_t step,
                            uint32_t ordinal, float sr_bias, float sr_eps,
                            int32_t device, void* stream);

int32_t aw4_dequantize_blocks(const aw4_scheme* scheme, const uint8_t* codes,
                              const float* scales, int64_t numel, float* out,
                              int32_t device, void* stream);

/* Nibble packing of one-code-per-byte arrays (any numel; odd tail padded). */
int32_t aw4_pack_codes(const uint8_t* codes, int64_t numel, uint8_t* packed,
                       int32_t device, void* stream);
int32_t aw4_unpack_codes(const uint8_t* packed, int64_t numel, uint8_t* codes,
                         int32_t device, void* stream);

/* Reads the sum over ranks of a gradient buffer through its NVLink multicast
 * address (multimem.ld_reduce, the same reduction as grad_multicast) and
 * writes out[i] = f32(sum[i]) * scale.  numel a multiple of 8; mc 16-byte
 * aligned; dtype AW4_F32, AW4_BF16 or AW4_F16.  ZeRO-2 uses it for the
 * tensors that keep FP32 moments.  No reference counterpart: the reference
 * has no data parallelism. */
int32_t aw4_reduce_multicast(const void* mc, int32_t dtype, int64_t numel, float scale,
                             float* out, int32_t device, void* stream);

/* Exhaustive device check of the reciprocal and square root the step kernel
 * builds from the hardware approximations, against IEEE round-to-nearest, over
 * every float32 of their domains (about 4e9 inputs each, a few ms).
 * counts: device pointer to 2 uint64, zeroed here, receiving the mismatch
 * counts [reciprocal, square root].  No reference counterpart: it validates
 * this build's arithmetic on the running GPU. */
int32_t aw4_selfcheck_math(uint64_t* counts, int32_t device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ADAMW4BIT_B200_H */
