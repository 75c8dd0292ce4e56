/*
 * fl_repack.cpp — raw GGUF blocks → device unit layout (fl_layout.h), and the
 * host emulation of the matvec kernel's arithmetic.
 *
 * Element accessors follow src/DotNetFoundryLLM.Quantization/Dequantizer.cs:
 * Q4_K nibble of byte e>>1 (:285-290), Q5_K high bit qh[e>>3] bit e&7
 * (:353-363), Q6_K ql nibble + 2 bits of qh[e>>2] at 2*(e&3) (:404-414), Q4_0
 * low nibble = element j, high nibble = element j+16 (:178-183).  A GGUF
 * tensor is one flat block stream (GgufModelLoader.cs:414-416), so row r of a
 * rows x cols matrix is flat elements [r*cols, (r+1)*cols).
 */
#include "fl_repack.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "fl_decode.h"

namespace {

int src_block_elems(int t)
{
    switch (t) {
    case FL_T_Q4_0: case FL_T_Q8_0: return 32;
    case FL_T_Q4_K: case FL_T_Q5_K: case FL_T_Q6_K: case FL_T_Q8_K: return 256;
    default: return 0;
    }
}
int src_block_bytes(int t)
{
    switch (t) {
    case FL_T_Q4_0: return 18;
    case FL_T_Q8_0: return 34;
    case FL_T_Q4_K: return 144;
    case FL_T_Q5_K: return 176;
    case FL_T_Q6_K: return 210;
    case FL_T_Q8_K: return 292;
    default: return 0;
    }
}

inline uint16_t ld16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

struct Src {
    int type, be, bb;
    const uint8_t* raw;
    const uint8_t* blk(int64_t f) const { return raw + (f / be) * bb; }
    /* raw quant of flat element f: unsigned level for the nibble formats,
     * signed int8 for Q8_0/Q8_K */
    int q(int64_t f) const
    {
        const uint8_t* b = blk(f);
        int e = (int)(f % be);
        switch (type) {
        case FL_T_Q4_K: return (b[16 + (e >> 1)] >> ((e & 1) * 4)) & 0xF;
        case FL_T_Q5_K: {
            int lo = (b[48 + (e >> 1)] >> ((e & 1) * 4)) & 0xF;
            int hi = (b[16 + (e >> 3)] >> (e & 7)) & 1;
            return lo | (hi << 4);
        }
        case FL_T_Q6_K: {
            int lo = (b[e >> 1] >> ((e & 1) * 4)) & 0xF;
            int hi = (b[128 + (e >> 2)] >> ((e & 3) * 2)) & 3;
            return lo | (hi << 4);
        }
        case FL_T_Q4_0: return e < 16 ? (b[2 + e] & 0xF) : (b[2 + e - 16] >> 4);
        case FL_T_Q8_0: return (int8_t)b[2 + e];
        default: return (int8_t)b[4 + e]; /* Q8_K */
        }
    }
    /* (mul, sub) of the 16 values starting at flat element f (f % 16 == 0) */
    void mulsub(int64_t f, float* mul, float* sub) const
    {
        const uint8_t* b = blk(f);
        int e = (int)(f % be);
        switch (type) {
        case FL_T_Q4_K:
        case FL_T_Q5_K: {
            int sc, mn;
            fl_kscale_min(b + 4, e / 32, &sc, &mn);
            *mul = fl_half_to_float(ld16(b)) * (float)sc;
            *sub = fl_half_to_float(ld16(b + 2)) * (float)mn;
            break;
        }
        case FL_T_Q6_K: {
            float m = fl_half_to_float(ld16(b + 208)) * (float)(int8_t)b[192 + e / 16];
            *mul = m;
            *sub = 32.0f * m;
            break;
        }
        case FL_T_Q4_0: {
            float d = fl_half_to_float(ld16(b));
            *mul = d;
            *sub = 8.0f * d;
            break;
        }
        case FL_T_Q8_0: *mul = fl_half_to_float(ld16(b)); *sub = 0.0f; break;
        default: { float d; memcpy(&d, b, 4); *mul = d; *sub = 0.0f; break; }
        }
    }
};

int fmt_of(int t)
{
    switch (t) {
    case FL_T_Q4_K: return FL_FMT_Q4K;
    case FL_T_Q5_K: return FL_FMT_Q5K;
    case FL_T_Q6_K: return FL_FMT_Q6K;
    case FL_T_Q8_0: return FL_FMT_Q8_0;
    case FL_T_Q4_0: return FL_FMT_Q4_0;
    case FL_T_Q8_K: return FL_FMT_Q8K;
    default: return -1;
    }
}

void repack_tiles(const fl_matrix_layout* L, const uint8_t* raw, const uint8_t* raw2, const int32_t* row_map,
                  uint8_t* dst, int t0, int t1)
{
    Src S1{L->ggml_type, src_block_elems(L->ggml_type), src_block_bytes(L->ggml_type), raw};
    Src S2{L->ggml_type, S1.be, S1.bb, raw2 ? raw2 : raw};
    fl_unit_off o = fl_offsets(L->fmt, L->expanded);
    const int64_t cols = L->cols;
    for (int T = t0; T < t1; T++) {
        const Src* src[16];
        int64_t rbase[16];
        bool valid[16];
        for (int r = 0; r < 16; r++) {
            int row = T * 16 + r;
            valid[r] = row < L->rows;
            int sr = valid[r] ? (row_map ? row_map[row] : row) : 0;
            src[r] = sr >= 0 ? &S1 : &S2;
            rbase[r] = (int64_t)(sr >= 0 ? sr : (-1 - sr)) * cols;
        }
        for (int kb = 0; kb < L->n_kb; kb++) {
            uint8_t* u = dst + ((int64_t)T * L->n_kb + kb) * L->unit_bytes;
            memset(u, 0, (size_t)L->unit_bytes);
            /* chunk validity: chunk c covers columns kb*256 + 32c .. +32 */
            auto chunk_ok = [&](int c) { return (int64_t)kb * 256 + 32 * c < cols; };
            /* headers */
            for (int r = 0; r < 16; r++) {
                if (!valid[r]) continue;
                const Src& s = *src[r];
                if (L->expanded) {
                    for (int c = 0; c < 8; c++) {
                        if (!chunk_ok(c)) continue;
                        for (int h = 0; h < 2; h++) {
                            float v[2];
                            s.mulsub(rbase[r] + (int64_t)kb * 256 + 32 * c + 16 * h, &v[0], &v[1]);
                            memcpy(u + ((r * 8 + c) * 2 + h) * 8, v, 8);
                        }
                    }
                    continue;
                }
                switch (L->fmt) {
                case FL_FMT_Q4K:
                case FL_FMT_Q5K: memcpy(u + r * 16, s.blk(rbase[r] + (int64_t)kb * 256), 16); break;
                case FL_FMT_Q6K: {
                    const uint8_t* b = s.blk(rbase[r] + (int64_t)kb * 256);
                    memcpy(u + FL_Q6K_SC + r * 16, b + 192, 16);
                    memcpy(u + FL_Q6K_D + r * 2, b + 208, 2);
                    break;
                }
                case FL_FMT_Q8_0:
                case FL_FMT_Q4_0:
                    for (int c = 0; c < 8; c++)
                        if (chunk_ok(c)) memcpy(u + (r * 8 + c) * 2, s.blk(rbase[r] + (int64_t)kb * 256 + 32 * c), 2);
                    break;
                default: memcpy(u + r * 4, s.blk(rbase[r] + (int64_t)kb * 256), 4); break;
                }
            }
            /* quant words, step s, lane l, word j = (chunk 2s + (j>>1), row g + 8(j&1)) */
            for (int s = 0; s < 4; s++)
                for (int l = 0; l < 32; l++) {
                    int g = l >> 2, t = l & 3;
                    uint32_t H = 0, H6[2] = {0, 0};
                    for (int j = 0; j < 4; j++) {
                        int c = 2 * s + (j >> 1), r = g + 8 * (j & 1);
                        int vals[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                        if (valid[r] && chunk_ok(c)) {
                            int64_t f0 = rbase[r] + (int64_t)kb * 256 + 32 * c + 8 * t;
                            for (int i = 0; i < 8; i++) vals[i] = src[r]->q(f0 + i);
                        }
                        if (fl_fmt_nibbles(L->fmt)) {
                            uint32_t w = 0;
                            for (int i = 0; i < 8; i++) w |= (uint32_t)(vals[i] & 0xF) << (4 * i);
                            memcpy(u + o.qs + ((s * 32 + l) * 4 + j) * 4, &w, 4);
                            for (int i = 0; i < 8; i++) {
                                int k = i >> 1, p = i & 1;
                                if (L->fmt == FL_FMT_Q5K)
                                    H |= (uint32_t)((vals[i] >> 4) & 1) << (8 * k + 2 * j + p);
                                if (L->fmt == FL_FMT_Q6K)
                                    H6[j >> 1] |= (uint32_t)((vals[i] >> 4) & 3) << (8 * k + 2 * (2 * (j & 1) + p));
                            }
                        } else {
                            uint8_t b8[8];
                            for (int k = 0; k < 4; k++) {
                                b8[k] = (uint8_t)(int8_t)vals[2 * k];
                                b8[4 + k] = (uint8_t)(int8_t)vals[2 * k + 1];
                            }
                            memcpy(u + o.qs + (((s * 2 + (j >> 1)) * 32 + l) * 16) + (j & 1) * 8, b8, 8);
                        }
                    }
                    if (L->fmt == FL_FMT_Q5K) memcpy(u + o.qh + (s * 32 + l) * 4, &H, 4);
                    if (L->fmt == FL_FMT_Q6K) memcpy(u + o.qh + (s * 32 + l) * 8, H6, 8);
                }
        }
    }
}

} // namespace

extern "C" int fl_layout_for(int32_t ggml_type, int32_t rows, int32_t cols, fl_matrix_layout* out)
{
    int fmt = fmt_of(ggml_type);
    if (fmt < 0) return -1;
    if (rows <= 0 || cols <= 0 || cols % 32 != 0) return -2;
    fl_matrix_layout L;
    memset(&L, 0, sizeof L);
    L.ggml_type = ggml_type;
    L.fmt = fmt;
    L.expanded = (src_block_elems(ggml_type) == 256 && cols % 256 != 0) ? 1 : 0;
    L.rows = rows;
    L.cols = cols;
    L.n_tiles = (rows + 15) / 16;
    L.n_kb = (cols + 255) / 256;
    fl_unit_off o = fl_offsets(fmt, L.expanded);
    L.unit_bytes = o.unit;
    L.hdr_bytes = o.hdr;
    L.total_bytes = (int64_t)L.n_tiles * L.n_kb * L.unit_bytes;
    L.gguf_bytes = (int64_t)rows * cols / src_block_elems(ggml_type) * src_block_bytes(ggml_type);
    *out = L;
    return 0;
}

extern "C" int fl_repack(const fl_matrix_layout* L, const uint8_t* raw, const uint8_t* raw2, const int32_t* row_map,
                         uint8_t* dst, int n_threads)
{
    if (n_threads <= 0) n_threads = (int)std::max(1u, std::thread::hardware_concurrency());
    n_threads = std::min(n_threads, L->n_tiles);
    if (n_threads <= 1) {
        repack_tiles(L, raw, raw2, row_map, dst, 0, L->n_tiles);
        return 0;
    }
    std::vector<std::thread> th;
    for (int i = 0; i < n_threads; i++) {
        int t0 = (int)((int64_t)L->n_tiles * i / n_threads), t1 = (int)((int64_t)L->n_tiles * (i + 1) / n_threads);
        th.emplace_back(repack_tiles, L, raw, raw2, row_map, dst, t0, t1);
    }
    for (auto& t : th) t.join();
    return 0;
}

/* Host twin of the kernel: x encoding (3 limbs, global scale absmax/127) and
 * the per-(row, chunk, half, limb) integer sums, then the epilogue formula. */
extern "C" int fl_emulate_matvec(const fl_matrix_layout* L, const uint8_t* packed, const float* x, float* y)
{
    const int K = L->n_kb * 256;
    std::vector<float> xp((size_t)K, 0.0f);
    memcpy(xp.data(), x, sizeof(float) * (size_t)L->cols);
    float amax = 0.0f;
    for (int i = 0; i < L->cols; i++) amax = std::max(amax, std::fabs(xp[i]));
    float s = amax / 127.0f;
    float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    std::vector<int> X[3];
    for (auto& v : X) v.assign((size_t)K, 0);
    const float inv14 = inv * 16384.0f;
    for (int i = 0; i < K; i++) {
        /* Y = rint(x * inv * 2^14) in one rounding (the device's FMA against
         * 1.5 * 2^23), cut into X0 * 2^14 + X1 * 2^7 + X2 */
        const int Y = (int)std::nearbyint((double)xp[i] * (double)inv14);
        const int x0 = (Y + 8192) >> 14;
        const int r = Y - x0 * 16384;
        const int x1 = (r + 64) >> 7;
        X[0][i] = x0;
        X[1][i] = x1;
        X[2][i] = r - x1 * 128;
    }
    std::vector<float> sx((size_t)K / 16, 0.0f);
    for (int i = 0; i < K / 16; i++) {
        float a = 0.0f;
        for (int k = 0; k < 16; k++) a += xp[i * 16 + k];
        sx[i] = a;
    }
    const float w_pair[2] = {1.0f / 128.0f, 1.0f / 2097152.0f};
    for (int T = 0; T < L->n_tiles; T++) {
        double dummy = 0;
        (void)dummy;
        float acc[16][2][2] = {}, minacc[16][2] = {};
        for (int kb = 0; kb < L->n_kb; kb++) {
            const uint8_t* u = packed + ((int64_t)T * L->n_kb + kb) * L->unit_bytes;
            for (int c = 0; c < 8; c++) {
                /* rebuild A (16 rows x 32 k-slots) from the lane fragments */
                int A[16][32];
                for (int l = 0; l < 32; l++) {
                    uint32_t a[4];
                    fl_unit_afrag(u, L->fmt, L->expanded, c, l, a);
                    int g = l >> 2, t = l & 3;
                    for (int b = 0; b < 4; b++) {
                        int v0 = (int)((a[0] >> (8 * b)) & 0xFF), v1 = (int)((a[1] >> (8 * b)) & 0xFF);
                        int v2 = (int)((a[2] >> (8 * b)) & 0xFF), v3 = (int)((a[3] >> (8 * b)) & 0xFF);
                        if (fl_fmt_signed(L->fmt)) { v0 = (int8_t)v0; v1 = (int8_t)v1; v2 = (int8_t)v2; v3 = (int8_t)v3; }
                        A[g][4 * t + b] = v0;
                        A[g + 8][4 * t + b] = v1;
                        A[g][16 + 4 * t + b] = v2;
                        A[g + 8][16 + 4 * t + b] = v3;
                    }
                }
                /* k-slot 4t+b ↔ value 8t+2b; slot 16+4t+b ↔ value 8t+2b+1 */
                int xk[3][32];
                for (int t = 0; t < 4; t++)
                    for (int b = 0; b < 4; b++)
                        for (int li = 0; li < 3; li++) {
                            int base = kb * 256 + 32 * c + 8 * t;
                            xk[li][4 * t + b] = X[li][base + 2 * b];
                            xk[li][16 + 4 * t + b] = X[li][base + 2 * b + 1];
                        }
                for (int r = 0; r < 16; r++)
                    for (int h = 0; h < 2; h++) {
                        int D[3] = {0, 0, 0};
                        for (int k = 0; k < 32; k++) {
                            int t = (k & 15) >> 2; /* word of slot k */
                            if ((t >> 1) != h) continue;
                            for (int li = 0; li < 3; li++) D[li] += A[r][k] * xk[li][k];
                        }
                        float mul, sub;
                        fl_unit_scale(u, L->fmt, L->expanded, r, c, h, &mul, &sub);
                        int ia = D[0] * 128 + D[1], ib = D[2] * 128;
                        acc[r][h][0] += (float)ia * mul;
                        acc[r][h][1] += (float)ib * mul;
                        minacc[r][h] += sub * sx[(kb * 256 + 32 * c) / 16 + h];
                    }
            }
        }
        for (int r = 0; r < 16; r++) {
            int row = T * 16 + r;
            if (row >= L->rows) continue;
            float lanes[4];
            for (int t = 0; t < 4; t++) {
                int h = t >> 1, p = t & 1;
                lanes[t] = acc[r][h][p] * (w_pair[p] * s) - (p == 0 ? minacc[r][h] : 0.0f);
            }
            y[row] = (lanes[0] + lanes[1]) + (lanes[2] + lanes[3]);
        }
    }
    return 0;
}
