/*
 * Oracle restatement of the reference's packed GEMV kernels — TEST
 * INFRASTRUCTURE ONLY (the CUDA library never links or calls this file).
 *
 * Restates, in plain scalar C99 (+ OpenMP across output rows), the
 * arithmetic of rwkv_ssd/native/lut2_gather.c in the reference engine:
 *
 *   oracle_sg8_gemv            <- scale_u8_grouped_row / _gemv_f32      (lut2_gather.c:336-496)
 *   oracle_lut2_grouped_gemv   <- trinity_grouped_lut2_gemv_f32         (lut2_gather.c:264-326)
 *   oracle_sg8_transposed_gemv <- scalar path of scale_u8_grouped_transposed_gemv_f32
 *                                                                       (lut2_gather.c:879-937)
 *   oracle_sg8_tmix_adapters   <- scale_u8_grouped_transposed_tmix_fused_f32_export
 *                                                                       (lut2_gather.c:1006-1103)
 *   oracle_sg8_cmix            <- scale_u8_grouped_cmix_gemv_f32        (lut2_gather.c:505-596)
 *   oracle_sg8_tmix_qkv        <- scale_u8_grouped_tmix_gemv_f32_n      (lut2_gather.c:1351-1399)
 *
 * Blobs are the raw wire bytes (header parsed here).  The SG8 GEMV uses the
 * reference's per-group algebra  acc += min*sum(x) + (max-min)/255*sum(q*x).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static uint32_t rd_u32(const uint8_t* p) { uint32_t v; memcpy(&v, p, 4); return v; }
static uint16_t rd_u16(const uint8_t* p) { uint16_t v; memcpy(&v, p, 2); return v; }
static float rd_f32(const uint8_t* p) { float v; memcpy(&v, p, 4); return v; }

/* IEEE binary16 -> binary32 (exact). */
static float half_to_float(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t m = (uint32_t)h & 0x3FFu;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int s = 0;
            while ((m & 0x400u) == 0) { m <<= 1; ++s; }
            m &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - s) << 23) | (m << 13);
        }
    } else if (e == 0x1Fu) {
        bits = sign | 0x7F800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f; memcpy(&f, &bits, 4); return f;
}

static float sg8_row(const uint8_t* scales, const uint8_t* quant, const float* x,
                     int in_f, uint32_t g, size_t row_base) {
    const float inv255 = 1.0f / 255.0f;
    size_t col = 0, logical = row_base;
    float acc = 0.0f;
    while (col < (size_t)in_f) {
        size_t grp = logical / g;
        size_t take = (grp + 1u) * g - logical;
        if (take > (size_t)in_f - col) take = (size_t)in_f - col;
        float sx = 0.0f, sqx = 0.0f;
        for (size_t j = 0; j < take; ++j) {
            float xv = x[col + j];
            sx += xv;
            sqx += (float)quant[logical + j] * xv;
        }
        float mn = rd_f32(scales + grp * 8u), mx = rd_f32(scales + grp * 8u + 4u);
        acc += mn * sx + (mx - mn) * inv255 * sqx;
        col += take;
        logical += take;
    }
    return acc;
}

int oracle_sg8_gemv(float* y, const uint8_t* blob, const float* x, int out_f, int in_f) {
    uint32_t g = rd_u32(blob + 4);
    if (g == 0) return 1;
    size_t n = (size_t)out_f * (size_t)in_f;
    size_t groups = (n + g - 1u) / g;
    const uint8_t* scales = blob + 8;
    const uint8_t* quant = scales + groups * 8u;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < out_f; ++r)
        y[r] = sg8_row(scales, quant, x, in_f, g, (size_t)r * (size_t)in_f);
    return 0;
}

int oracle_sg8_tmix_qkv(float* y, const uint8_t* const* blobs, const float* const* xs,
                        int out_f, int in_f, int n_mats) {
    for (int m = 0; m < n_mats; ++m) {
        int rc = oracle_sg8_gemv(y + (size_t)m * out_f, blobs[m], xs[m], out_f, in_f);
        if (rc) return rc;
    }
    return 0;
}

int oracle_lut2_grouped_gemv(float* y, const uint8_t* blob, const float* x, int out_f, int in_f) {
    uint8_t kind = blob[3];
    uint32_t g = rd_u32(blob + 4);
    if (g == 0) return 1;
    size_t n = (size_t)out_f * (size_t)in_f;
    size_t groups = (n + g - 1u) / g;
    int input_layout = (kind == 6 || kind == 7);
    int residual = (kind == 5 || kind == 7);
    int fp32_cb = (kind == 3);
    size_t rec = residual ? 16u : (fp32_cb ? 16u : 8u);
    const uint8_t* records = blob + 8;
    const uint8_t* packed = records + groups * rec;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < out_f; ++r) {
        float acc = 0.0f;
        for (int c = 0; c < in_f; ++c) {
            size_t logical = input_layout ? (size_t)c * (size_t)out_f + (size_t)r
                                          : (size_t)r * (size_t)in_f + (size_t)c;
            size_t grp = logical / g, local = logical % g;
            unsigned code = (packed[logical >> 2] >> ((logical & 3u) * 2u)) & 3u;
            const uint8_t* rc = records + grp * rec;
            float w = fp32_cb ? rd_f32(rc + code * 4u) : half_to_float(rd_u16(rc + code * 2u));
            if (residual) {
                if (local == rc[8]) w += half_to_float(rd_u16(rc + 10));
                else if (local == rc[9]) w += half_to_float(rd_u16(rc + 12));
            }
            acc += w * x[c];
        }
        y[r] = acc;
    }
    return 0;
}

/* y = x @ W for a row-major [in_f, out_f] SG8 blob (compact TMix adapters). */
int oracle_sg8_transposed_gemv(float* y, const uint8_t* blob, const float* x, int out_f, int in_f) {
    uint32_t g = rd_u32(blob + 4);
    if (g == 0) { memset(y, 0, (size_t)out_f * sizeof(float)); return 1; }
    size_t n = (size_t)out_f * (size_t)in_f;
    size_t groups = (n + g - 1u) / g;
    const uint8_t* scales = blob + 8;
    const uint8_t* quant = scales + groups * 8u;
    const float inv255 = 1.0f / 255.0f;
#pragma omp parallel for schedule(static)
    for (int c = 0; c < out_f; ++c) {
        float acc = 0.0f;
        for (int r = 0; r < in_f; ++r) {
            size_t logical = (size_t)r * (size_t)out_f + (size_t)c;
            size_t grp = logical / g;
            float mn = rd_f32(scales + grp * 8u), mx = rd_f32(scales + grp * 8u + 4u);
            float w = mn + (mx - mn) * ((float)quant[logical] * inv255);
            acc += w * x[r];
        }
        y[c] = acc;
    }
    return 0;
}

/* blobs: w1,w2,a1,a2,g1,g2,v1,v2 ; xs: xw,xa,xg,xv ; ranks: w,a,g,v */
int oracle_sg8_tmix_adapters(float* w_out, float* a_out, float* g_out, float* v_out,
                             const uint8_t* const* blobs, const float* const* xs,
                             const float* a0, int C, const int* ranks, int has_v) {
    int rw = ranks[0], ra = ranks[1], rg = ranks[2], rv = has_v ? ranks[3] : 0;
    float* mid = (float*)malloc((size_t)(rw + ra + rg + rv) * sizeof(float));
    if (!mid) return 2;
    float *wm = mid, *am = wm + rw, *gm = am + ra, *vm = gm + rg;
    oracle_sg8_transposed_gemv(wm, blobs[0], xs[0], rw, C);
    oracle_sg8_transposed_gemv(am, blobs[2], xs[1], ra, C);
    oracle_sg8_transposed_gemv(gm, blobs[4], xs[2], rg, C);
    if (has_v) oracle_sg8_transposed_gemv(vm, blobs[6], xs[3], rv, C);
    for (int i = 0; i < rw; ++i) wm[i] = tanhf(wm[i]);
    for (int i = 0; i < rg; ++i) gm[i] = 1.0f / (1.0f + expf(-gm[i]));
    oracle_sg8_transposed_gemv(w_out, blobs[1], wm, C, rw);
    oracle_sg8_transposed_gemv(a_out, blobs[3], am, C, ra);
    oracle_sg8_transposed_gemv(g_out, blobs[5], gm, C, rg);
    if (has_v) oracle_sg8_transposed_gemv(v_out, blobs[7], vm, C, rv);
    for (int i = 0; i < C; ++i) {
        float b = a0 ? a0[i] : 0.0f;
        a_out[i] = 1.0f / (1.0f + expf(-(b + a_out[i])));
    }
    free(mid);
    return 0;
}

/* y = Wv @ relu(Wk @ x)^2 */
int oracle_sg8_cmix(float* y, const uint8_t* key_blob, const uint8_t* value_blob, const float* x,
                    int ko, int ki, int vo, int vi) {
    if (ko <= 0 || ki <= 0 || vo <= 0 || vi != ko) return 1;
    float* h = (float*)malloc((size_t)ko * sizeof(float));
    if (!h) return 2;
    int rc = oracle_sg8_gemv(h, key_blob, x, ko, ki);
    if (rc) { free(h); return rc; }
    for (int i = 0; i < ko; ++i) h[i] = h[i] > 0.0f ? h[i] * h[i] : 0.0f;
    rc = oracle_sg8_gemv(y, value_blob, h, vo, vi);
    free(h);
    return rc;
}

/* Per-tensor LUT2 (TR2\x01: magic, fp32 codebook[4], 2-bit codes LSB first):
   y = W @ x with the row walk of lut2_gemv_f32 (lut2_gather.c:179-211) -- row r
   reads its codes from byte (r * in) / 4 on, four per byte; per byte the four
   products are summed, then added to the row total. */
int oracle_lut2_tensor_gemv(float* y, const uint8_t* blob, const float* x, int out_f, int in_f) {
    if (out_f <= 0 || in_f <= 0 || memcmp(blob, "TR2\x01", 4) != 0) return 1;
    float cb[4];
    for (int k = 0; k < 4; ++k) cb[k] = rd_f32(blob + 4 + 4 * k);
    const uint8_t* packed = blob + 20;
#pragma omp parallel for schedule(static)
    for (int row = 0; row < out_f; ++row) {
        const uint8_t* prow = packed + (((size_t)row * (size_t)in_f) >> 2);
        float acc = 0.0f;
        int col = 0;
        for (; col + 4 <= in_f; col += 4) {
            const uint8_t b = *prow++;
            acc += cb[b & 3u] * x[col] + cb[(b >> 2) & 3u] * x[col + 1] + cb[(b >> 4) & 3u] * x[col + 2] +
                   cb[(b >> 6) & 3u] * x[col + 3];
        }
        if (col < in_f) {
            const uint8_t b = *prow;
            for (int shift = 0; col < in_f; ++col, shift += 2) acc += cb[(b >> shift) & 3u] * x[col];
        }
        y[row] = acc;
    }
    return 0;
}

/* Activation-INT8 SG8 GEMV (lut2_gather.c:612-796): per input group, scale =
   max|x| / 127 (1 when max|x| <= 1e-12), q = x * (1 / scale) rounded half away
   from zero, clamped to +-127, sum(x) in column order; per row and group
   min * sum(x) + (max - min) / 255 * scale * sum(q_w * q_x) with an exact
   integer dot.  A row width that is not a multiple of the group falls back
   to the float GEMV, as the reference does. */
int oracle_sg8_i8_gemv(float* y, const uint8_t* blob, const float* x, int out_f, int in_f) {
    if (memcmp(blob, "SG8\x01", 4) != 0 || out_f <= 0 || in_f <= 0) return 1;
    const uint32_t g = rd_u32(blob + 4);
    if (g == 0u || (in_f % (int)g) != 0) return oracle_sg8_gemv(y, blob, x, out_f, in_f);
    const int groups = in_f / (int)g;
    int8_t* q = (int8_t*)malloc((size_t)in_f);
    float* scale = (float*)malloc((size_t)groups * sizeof(float));
    float* sum_x = (float*)malloc((size_t)groups * sizeof(float));
    if (!q || !scale || !sum_x) { free(q); free(scale); free(sum_x); return 2; }
    for (int gi = 0; gi < groups; ++gi) {
        const int b0 = gi * (int)g, b1 = b0 + (int)g;
        float m = 0.0f, s = 0.0f;
        for (int c = b0; c < b1; ++c) {
            const float a = x[c] < 0.0f ? -x[c] : x[c];
            if (a > m) m = a;
            s += x[c];
        }
        const float sc = m > 1.0e-12f ? m / 127.0f : 1.0f;
        const float inv = 1.0f / sc;
        scale[gi] = sc;
        sum_x[gi] = s;
        for (int c = b0; c < b1; ++c) {
            const float v = x[c] * inv;
            int qi = v >= 0.0f ? (int)(v + 0.5f) : (int)(v - 0.5f);
            qi = qi > 127 ? 127 : (qi < -127 ? -127 : qi);
            q[c] = (int8_t)qi;
        }
    }
    const size_t n = (size_t)out_f * (size_t)in_f;
    const size_t ngroups = (n + g - 1u) / g;
    const uint8_t* scales = blob + 8;
    const uint8_t* quant = scales + ngroups * 8u;
#pragma omp parallel for schedule(static)
    for (int row = 0; row < out_f; ++row) {
        const size_t rg = (size_t)row * (size_t)groups;
        float acc = 0.0f;
        for (int gi = 0; gi < groups; ++gi) {
            const uint8_t* wq = quant + (rg + (size_t)gi) * g;
            int32_t dot = 0;
            for (uint32_t c = 0; c < g; ++c) dot += (int32_t)wq[c] * (int32_t)q[(size_t)gi * g + c];
            const float mn = rd_f32(scales + (rg + (size_t)gi) * 8u);
            const float mx = rd_f32(scales + (rg + (size_t)gi) * 8u + 4u);
            acc += mn * sum_x[gi] + (mx - mn) * (1.0f / 255.0f) * scale[gi] * (float)dot;
        }
        y[row] = acc;
    }
    free(q);
    free(scale);
    free(sum_x);
    return 0;
}
