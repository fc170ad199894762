/*
 * m27b_blocks.h — GGUF k-quant block layouts consumed by the quantized matvec
 * path, byte for byte as the reference declares them:
 *
 *   m27b_block_q4_K   <- BlockQ4K    src/mono27b_executor.cu:18-23   (144 B)
 *   m27b_block_q8_0   <- BlockQ8     src/mono27b_executor.cu:25-28   ( 34 B)
 *   m27b_block_q5_K   <- BlockQ5K    src/mono27b_executor.cu:30-36   (176 B)
 *   m27b_block_q8_K   <- BlockQ8K    src/mono27b_executor.cu:38-42   (292 B)
 *   m27b_block_iq4_xs <- BlockIQ4XS  src/mono27b_executor.cu:44-49   (136 B)
 *   m27b_block_q6_K   <- BlockQ6K    src/mono27b_executor.cu:57-62   (210 B)
 *
 * The ggml type codes are the reference's Mono27BGgmlType values
 * (include/mono27b_gguf.h:28-44).  fp16 fields are carried as raw uint16 bits
 * so that this header is plain C and usable from host code without CUDA.
 */
#ifndef M27B_BLOCKS_H
#define M27B_BLOCKS_H

#include <stdint.h>

#define M27B_TYPE_F32 0u
#define M27B_TYPE_F16 1u
#define M27B_TYPE_Q8_0 8u
#define M27B_TYPE_Q4_K 12u
#define M27B_TYPE_Q5_K 13u
#define M27B_TYPE_Q6_K 14u
#define M27B_TYPE_Q8_K 15u
#define M27B_TYPE_IQ4_XS 23u

/* Layout flag OR-ed into WeightView.ggml_type for tensors repacked at load
 * time into the planar row layout (see m27b_qmv.h, m27b_repack). */
#define M27B_LAYOUT_PLANAR 0x100u
#define M27B_TYPE_MASK 0xffu

#define M27B_QK_K 256
#define M27B_QK8_0 32

typedef struct {
    uint16_t d;          /* fp16 super-block scale of the 6-bit sub-scales */
    uint16_t dmin;       /* fp16 super-block scale of the 6-bit sub-mins   */
    uint8_t scales[12];  /* 8 x (6-bit scale, 6-bit min), packed          */
    uint8_t qs[128];     /* 256 x 4-bit codes                             */
} m27b_block_q4_K;

typedef struct {
    uint16_t d;          /* fp16 super-block scale of the 6-bit sub-scales  */
    uint16_t dmin;       /* fp16 super-block scale of the 6-bit sub-mins    */
    uint8_t scales[12];  /* packed as in q4_K                               */
    uint8_t qh[32];      /* bit s of qh[l]: bit 4 of element l of sub-block s */
    uint8_t qs[128];     /* low 4 bits, nibble layout as in q4_K            */
} m27b_block_q5_K;

typedef struct {
    uint16_t d;          /* fp16 super-block scale                          */
    uint16_t scales_h;   /* 2 high bits of each sub-block's 6-bit scale     */
    uint8_t scales_l[4]; /* 4 low bits of each (two per byte)               */
    uint8_t qs[128];     /* sub-block i: qs[16i..16i+15], low nibbles first */
} m27b_block_iq4_xs;

typedef struct {
    uint8_t ql[128];     /* low 4 bits of 256 6-bit codes */
    uint8_t qh[64];      /* high 2 bits                   */
    int8_t scales[16];   /* one int8 scale per 16 values  */
    uint16_t d;          /* fp16 super-block scale        */
} m27b_block_q6_K;

typedef struct {
    uint16_t d;          /* fp16 scale */
    int8_t qs[32];
} m27b_block_q8_0;

typedef struct {
    float d;             /* fp32 scale (1/iscale; may be negative) */
    int8_t qs[256];
    int16_t bsums[16];   /* sum of each 16 consecutive codes */
} m27b_block_q8_K;

#ifdef __cplusplus
static_assert(sizeof(m27b_block_q4_K) == 144, "q4_K block must be 144 bytes");
static_assert(sizeof(m27b_block_q5_K) == 176, "q5_K block must be 176 bytes");
static_assert(sizeof(m27b_block_iq4_xs) == 136, "IQ4_XS block must be 136 bytes");
static_assert(sizeof(m27b_block_q6_K) == 210, "q6_K block must be 210 bytes");
static_assert(sizeof(m27b_block_q8_0) == 34, "q8_0 block must be 34 bytes");
static_assert(sizeof(m27b_block_q8_K) == 292, "q8_K block must be 292 bytes");
#else
_Static_assert(sizeof(m27b_block_q4_K) == 144, "q4_K block must be 144 bytes");
_Static_assert(sizeof(m27b_block_q5_K) == 176, "q5_K block must be 176 bytes");
_Static_assert(sizeof(m27b_block_iq4_xs) == 136, "IQ4_XS block must be 136 bytes");
_Static_assert(sizeof(m27b_block_q6_K) == 210, "q6_K block must be 210 bytes");
_Static_assert(sizeof(m27b_block_q8_0) == 34, "q8_0 block must be 34 bytes");
_Static_assert(sizeof(m27b_block_q8_K) == 292, "q8_K block must be 292 bytes");
#endif

#endif /* M27B_BLOCKS_H */
