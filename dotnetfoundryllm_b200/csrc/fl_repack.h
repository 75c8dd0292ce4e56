/*
 * fl_repack.h — host-side repack of raw GGUF blocks into the device unit
 * layout of fl_layout.h, plus a scalar emulation of the matvec kernel's
 * integer arithmetic used by the CPU tests.
 */
#ifndef FL_REPACK_H
#define FL_REPACK_H

#include <stddef.h>
#include <stdint.h>

#include "fl_layout.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct fl_matrix_layout {
    int32_t ggml_type;   /* source GGUF type */
    int32_t fmt;         /* FL_FMT_* */
    int32_t expanded;    /* 1 = per-chunk float headers (straddling rows) */
    int32_t rows, cols;  /* logical shape */
    int32_t n_tiles;     /* ceil(rows / 16) */
    int32_t n_kb;        /* ceil(cols / 256) */
    int32_t unit_bytes;  /* bytes of one (tile, k-block) unit */
    int32_t hdr_bytes;   /* header bytes at the start of a unit */
    int64_t total_bytes; /* n_tiles * n_kb * unit_bytes */
    int64_t gguf_bytes;  /* payload bytes of the GGUF tensor (rows*cols elements) */
} fl_matrix_layout;

/* Fills the layout for a rows x cols matrix of the given GGUF type.
 * Returns 0, or -1 when the type has no quantized matvec path (F32/F16/BF16
 * are handled by the float path), -2 when cols is not a multiple of 32. */
int fl_layout_for(int32_t ggml_type, int32_t rows, int32_t cols, fl_matrix_layout* out);

/* Repacks rows*cols elements of raw GGUF bytes into dst (total_bytes).
 * `row_map` (optional, rows entries) gives, for each device row, the source
 * row to read (used to interleave gate/up rows); NULL = identity.  The source
 * of device row r is `raw` when row_map[r] >= 0, `raw2` row (-1 - row_map[r])
 * otherwise.  n_threads <= 0 uses the hardware concurrency. */
int fl_repack(const fl_matrix_layout* L, const uint8_t* raw, const uint8_t* raw2, const int32_t* row_map,
              uint8_t* dst, int n_threads);

/* Scalar emulation of the device kernel on a repacked matrix: encodes x the
 * way the kernel prologue does (3 int8 limbs, scale absmax/127), forms the
 * per-(row, chunk, half, limb) integer sums the tensor core computes and
 * applies the same epilogue.  Used by the CPU tests to check the layout and
 * the arithmetic against the oracle without a GPU. */
int fl_emulate_matvec(const fl_matrix_layout* L, const uint8_t* packed, const float* x, float* y);

#ifdef __cplusplus
}
#endif
#endif
