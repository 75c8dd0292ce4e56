/*
 * fl_layout.h — device layout of repacked quantized matrices (host + device).
 *
 * A matrix of R rows x C columns (GGUF ne0 = C) is cut into tiles of 16 rows
 * (the M of the int8 tensor-core MMA) and k-blocks of 256 columns (8 chunks of
 * 32).  One (tile, k-block) pair is a UNIT; units are stored tile-major
 * (k-block fastest), so any contiguous unit range is one contiguous byte range
 * that a single bulk copy moves into shared memory.  Rows are zero-padded to a
 * multiple of 16 and columns to a multiple of 256.
 *
 * Inside a unit the quantized values are stored in MMA fragment order: lane
 * l = 4*g + t of a warp reads, for chunk c, the 8 values [32c+8t, 32c+8t+8) of
 * rows g and g+8 ("word" (c, t) of those rows).  Step s (0..3) holds chunks
 * 2s and 2s+1, so each lane reads one 16-byte vector per step and a warp reads
 * 512 contiguous bytes (no bank conflicts).  Within a step, word j (0..3) is
 * (chunk 2s + (j>>1), row g + 8*(j&1)).
 *
 * The nibble, high-bit and scale encodings are the reference's
 * (src/DotNetFoundryLLM.Quantization/Dequantizer.cs): a unit carries exactly
 * the bits of the 16 x 256 values it covers, rearranged, and the byte count of
 * a unit equals 16 GGUF blocks (Q4_K 2304, Q5_K 2816, Q6_K 3360, Q4_0 2304,
 * Q8_0 4352) — the device reads the GGUF payload once, no more.  Q8_K drops
 * its unused bsums (4160 bytes per unit).
 *
 * Rows whose GGUF blocks straddle row boundaries (C not a multiple of 256 for
 * the K-quants) use EXPANDED headers: one (mul, sub) float pair per row, chunk
 * and half-chunk, so v = mul*q - sub.
 */
#ifndef FL_LAYOUT_H
#define FL_LAYOUT_H

#include <stdint.h>

#define FL_TILE_ROWS 16
#define FL_KBLOCK 256
#define FL_CHUNKS 8

enum fl_ggml_type {
    FL_T_F32 = 0,
    FL_T_F16 = 1,
    FL_T_Q4_0 = 2,
    FL_T_Q8_0 = 8,
    FL_T_Q4_K = 12,
    FL_T_Q5_K = 13,
    FL_T_Q6_K = 14,
    FL_T_Q8_K = 15,
    FL_T_BF16 = 30,
};

/* Device formats of a repacked matrix (what the matvec kernel decodes). */
enum fl_fmt {
    FL_FMT_Q4K = 0,   /* u8 nibbles; header d,dmin,scales[12] per row: v = (d*sc)q - (dmin*m) */
    FL_FMT_Q5K = 1,   /* + 1 high bit per value */
    FL_FMT_Q6K = 2,   /* u8 0..63 (offset 32); int8 scale per 16 values, f16 d per row */
    FL_FMT_Q8_0 = 3,  /* s8; f16 d per chunk */
    FL_FMT_Q4_0 = 4,  /* u8 nibbles (offset 8); f16 d per chunk */
    FL_FMT_Q8K = 5,   /* s8; f32 d per row */
    FL_FMT_COUNT = 6,
};

/* Header-less "expanded" variants (straddling rows) share the quant layout of
 * the base format; the unit then starts with 16 rows x 8 chunks x 2 halves x
 * (mul, sub) floats = 2048 bytes of headers. */
#define FL_EXP_HDR_BYTES 2048

/* Byte offsets inside one unit, per format (compact headers). */
#define FL_Q4K_HDR 0        /* 16 rows x 16 B: d(f16) dmin(f16) scales[12] */
#define FL_Q4K_QS 256       /* 2048 B fragment-ordered nibble words */
#define FL_Q4K_UNIT 2304

#define FL_Q5K_HDR 0        /* 16 x 16 B as Q4_K */
#define FL_Q5K_QH 256       /* 512 B: one u32 per (step, lane), 1 bit per value */
#define FL_Q5K_QS 768       /* 2048 B nibble words */
#define FL_Q5K_UNIT 2816

#define FL_Q6K_SC 0         /* 16 rows x 16 int8 scales */
#define FL_Q6K_D 256        /* 16 rows x f16 d (32 B) */
#define FL_Q6K_QH 288       /* 1024 B: two u32 per (step, lane), 2 bits per value */
#define FL_Q6K_QL 1312      /* 2048 B nibble words */
#define FL_Q6K_UNIT 3360

#define FL_Q80_D 0          /* 16 rows x 8 chunks f16 d (256 B) */
#define FL_Q80_QS 256       /* 4096 B: [step][half][lane][16 B] byte-permuted words */
#define FL_Q80_UNIT 4352

#define FL_Q40_D 0          /* 16 x 8 f16 d */
#define FL_Q40_QS 256       /* 2048 B nibble words (sequential element order) */
#define FL_Q40_UNIT 2304

#define FL_Q8K_D 0          /* 16 rows x f32 d (64 B) */
#define FL_Q8K_QS 64        /* 4096 B as Q8_0 */
#define FL_Q8K_UNIT 4160

/* x-vector encoding in shared memory, per chunk of 32 inputs:
 *  - 3 int8 limbs (x ≈ s*(X0 + X1/128 + X2/16384)) in B-fragment order
 *    [limb][t][8 B] (4 bytes of even values then 4 bytes of odd values of word t);
 *  - [t] short2 limb sums of lane t's two MMA output columns over its half
 *    chunk: t even (S0, S1), t odd (S2, 0), half = t >> 1 (|S| <= 16*127);
 *  - [half] float sums of the 16 inputs of each half. */
#define FL_XENC_LIMB_BYTES 96
#define FL_XENC_LSUM_BYTES 16
#define FL_XENC_HSUM_BYTES 8
#define FL_XENC_CHUNK_BYTES (FL_XENC_LIMB_BYTES + FL_XENC_LSUM_BYTES + FL_XENC_HSUM_BYTES)
/* zero bytes read by lanes whose B column is not theirs (8 chunks apart) */
#define FL_XENC_ZERO_BYTES (8 * FL_XENC_LIMB_BYTES)

#endif
