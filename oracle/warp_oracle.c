/*
 * warp_oracle.c — TEST INFRASTRUCTURE: a CPU restatement of WARP's quantized
 * expert-FFN path, written from the reference's behaviour, used only as the
 * checker for the CUDA kernels (tests/, __graft_entry__.smoke, and bench.py's
 * cpu_baseline / reference arm).  The product never links or loads it.
 *
 * Parity is pinned: tests/test_oracle_vs_ref.py runs every function here
 * against the reference's own compiled code (oracle/_ref, built by
 * oracle/Makefile from the reference sources) on seeded inputs, and
 * tests/test_oracle_golden.py against the fixtures in tests/golden/, which
 * tests/golden/make_golden.py generated from the reference.
 *
 * Citations are path:line in the reference project.  Floating-point order is
 * the reference's wherever a function claims bit-exactness; the comments say
 * which order that is.  Build: plain gcc -O2 with no -mfma, so a*b+c is two
 * roundings exactly as in the reference's portable C.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define WO_VEC 8          /* vec_dim, convert.py:145                         */
#define WO_ENT 256        /* entries per stage, convert.py:146               */
#define WO_ST 3           /* VQ3R stages, waste_format.h:50                  */
#define WO_BLK 64         /* index_block, convert.py:148 / model.c:3890      */

/* ---- fp16 ------------------------------------------------------------------ */

/* waste_f16 (simd.h:81-99): fp16 -> fp32 keeping subnormals (mantissa*2^-24). */
float wo_f16(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1f, mn = h & 0x3ff;
    if (e == 0) {
        const float f = (float)mn * 5.9604644775390625e-08f;
        return sign ? -f : f;
    }
    const uint32_t bits = sign | ((e + 112u) << 23) | (mn << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* fp32 -> fp16, round to nearest even, subnormals and overflow handled: the
 * conversion torch's Tensor.half() performs on the converter's scales and
 * codebooks (convert.py:851, 910, 925, 1362).  Written from the IEEE 754
 * binary16 definition. */
uint16_t wo_f32_to_f16(float f)
{
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u)                          /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    if (ax >= 0x477ff000u)                          /* rounds to >= 65520 */
        return (uint16_t)(sign | 0x7c00u);
    const int e = (int)(ax >> 23) - 127;
    if (e >= -14) {                                 /* normal half */
        uint32_t m = ax & 0x7fffffu;
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
        const uint32_t rem = m & 0x1fffu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    if (e < -25) return (uint16_t)sign;             /* below half the min subnormal */
    /* subnormal half: value = m * 2^-24 */
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u; /* 24-bit significand */
    const int shift = -e - 14 + 13;                 /* bits to drop */
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* ---- codebooks --------------------------------------------------------------- */

/* The loader's decode (model.c:2911-2924): fp16 -> fp32 with subnormals
 * flushed to zero (unlike waste_f16), then the [book][dim][entry] transpose
 * (model.c:2929-2941). */
void wo_books_decode(const uint16_t *h, int n_books, float *books, float *booksT)
{
    const size_t per = (size_t)WO_ENT * WO_VEC;
    for (size_t i = 0; i < (size_t)n_books * per; i++) {
        const uint16_t v = h[i];
        const uint32_t sign = (uint32_t)(v >> 15) << 31;
        const uint32_t e = (v >> 10) & 0x1f, man = v & 0x3ff;
        const uint32_t bits = e ? (sign | ((e + 112u) << 23) | (man << 13)) : sign;
        memcpy(&books[i], &bits, 4);
    }
    if (booksT)
        for (int b = 0; b < n_books; b++)
            for (int c = 0; c < WO_ENT; c++)
                for (int d = 0; d < WO_VEC; d++)
                    booksT[(size_t)b * per + (size_t)d * WO_ENT + c] =
                        books[(size_t)b * per + (size_t)c * WO_VEC + d];
}

/* ---- VQ3R LUT build and apply ----------------------------------------------- */

/* lut[v][s][c] = sum_d x[8v+d] * C_{cb_base+s}[c][d], accumulated as the
 * dispatched x86 kernel does it: an FMA chain over d = 0..7 starting from 0
 * (lutb_range_avx512, simd_avx512.c:90-127; the AVX2 one is the same chain,
 * simd_avx2.c:100).  The portable waste_lutb_range (model.c:3815) uses
 * mul+add instead; wo_lut_build_muladd restates that one. */
void wo_lut_build(float *lut, const float *booksT, const float *x, int nv,
                  int cb_base)
{
    for (int v = 0; v < nv; v++)
        for (int s = 0; s < WO_ST; s++) {
            const float *CT = booksT + (size_t)(cb_base + s) * WO_ENT * WO_VEC;
            float *dst = lut + ((size_t)v * WO_ST + s) * WO_ENT;
            for (int c = 0; c < WO_ENT; c++) {
                float t = 0.0f;
                for (int d = 0; d < WO_VEC; d++)
                    t = fmaf(x[v * WO_VEC + d], CT[(size_t)d * WO_ENT + c], t);
                dst[c] = t;
            }
        }
}

void wo_lut_build_muladd(float *lut, const float *booksT, const float *x,
                         int nv, int cb_base)
{
    for (int v = 0; v < nv; v++)
        for (int s = 0; s < WO_ST; s++) {
            const float *CT = booksT + (size_t)(cb_base + s) * WO_ENT * WO_VEC;
            float *dst = lut + ((size_t)v * WO_ST + s) * WO_ENT;
            for (int c = 0; c < WO_ENT; c++) {
                float t = 0.0f;
                for (int d = 0; d < WO_VEC; d++) {
                    const float p = x[v * WO_VEC + d] * CT[(size_t)d * WO_ENT + c];
                    t = t + p;
                }
                dst[c] = t;
            }
        }
}

/* vq_rows (model.c:3909-3977): y[r] = (sum over v ascending of
 * ((T0[i0] + T1[i1]) + T2[i2])) * f16(scale[r]), indices read from the
 * blocked layout [M/64][nv][64 rows][3 stages] (FORMAT.md "Index layout is
 * blocked by 64 rows"; convert.py:777-792). */
void wo_vq_rows(float *y, const uint8_t *idx, const uint16_t *scale,
                const float *lut, int M, int nv)
{
    for (int r = 0; r < M; r++) {
        const int rb = r / WO_BLK, ri = r % WO_BLK;
        float acc = 0.0f;
        for (int v = 0; v < nv; v++) {
            const float *blk = lut + (size_t)v * WO_ST * WO_ENT;
            const uint8_t *ix = idx + (((size_t)rb * nv + v) * WO_BLK + ri) * WO_ST;
            const float t = (blk[ix[0]] + blk[WO_ENT + ix[1]]) + blk[2 * WO_ENT + ix[2]];
            acc += t;
        }
        y[r] = acc * wo_f16(scale[r]);
    }
}

/* ---- VQ4P: four stages of 64 entries, 6-bit packed (FORMAT.md "VQ4P record") */

/* The table build for any (stages, entries) geometry (lutb_range,
 * model.c:3815-3852, the same FMA chain over d from 0 as wo_lut_build):
 * lut[v][s][c] = sum_d x[8v+d] * booksT[cb_base+s][d][c], booksT of
 * `entries` columns. */
void wo_lut_build_se(float *lut, const float *booksT, const float *x, int nv, int cb_base,
                     int st, int en)
{
    for (int v = 0; v < nv; v++)
        for (int s = 0; s < st; s++) {
            const float *CT = booksT + (size_t)(cb_base + s) * en * WO_VEC;
            float *dst = lut + ((size_t)v * st + s) * en;
            for (int c = 0; c < en; c++) {
                float t = 0.0f;
                for (int d = 0; d < WO_VEC; d++)
                    t = fmaf(x[v * WO_VEC + d], CT[(size_t)d * en + c], t);
                dst[c] = t;
            }
        }
}

/* vq_quant_lut / vq_quant_range (model.c:3996-4068): per block of 32 vector
 * positions (WASTE_VQ_LUT_BLK, model.h:87), mx = max |lut| over the block's
 * entries, scale[blk] = mx / 127, inv = 127 / mx (0 when mx is 0), and
 * q = lrintf(lut * inv) clamped to [-127, 127]. */
void wo_vq_quant_lut(const float *lut, int nv, int st, int en, int8_t *q, float *scale)
{
    const int nblk = (nv + 31) / 32;
    for (int blk = 0; blk < nblk; blk++) {
        const int v0 = blk * 32;
        const int v1 = v0 + 32 < nv ? v0 + 32 : nv;
        const size_t n = (size_t)(v1 - v0) * st * en;
        const float *src = lut + (size_t)v0 * st * en;
        int8_t *dst = q + (size_t)v0 * st * en;
        float mx = 0.0f;
        for (size_t i = 0; i < n; i++) {
            const float f = fabsf(src[i]);
            if (f > mx) mx = f;
        }
        scale[blk] = mx / 127.0f;
        const float inv = mx > 0 ? 127.0f / mx : 0.0f;
        for (size_t i = 0; i < n; i++) {
            long t = lrintf(src[i] * inv);
            if (t > 127) t = 127;
            else if (t < -127) t = -127;
            dst[i] = (int8_t)t;
        }
    }
}

/* waste_vq_rows_p6 (model.c:4076-4113): the VQ4P apply.  Index bytes in the
 * blocked layout [M/64][nv][64 rows][3 bytes]; per row and vector position,
 * four 6-bit indices j0..j3 (b0 & 63; b0 >> 6 | b1 << 2; b1 >> 4 | b2 << 4;
 * b2 >> 2, each & 63: simd.h:73-76) into the int8 table T[v][4][64]; per
 * block of 32 positions the integer sum of the 4 lookups of every position,
 * then acc += lscale[blk] * sum in block order (fp32 multiply, then add), and
 * y[r] = acc * f16(scale[r]). */
void wo_vq_rows_p6(float *y, const uint8_t *idx, const uint16_t *scale, const int8_t *lut8,
                   const float *lscale, int M, int nv)
{
    for (int r = 0; r < M; r++) {
        const int rb = r / WO_BLK, ri = r % WO_BLK;
        float acc = 0.0f;
        for (int v0 = 0; v0 < nv; v0 += 32) {
            const int v1 = v0 + 32 < nv ? v0 + 32 : nv;
            int sum = 0;
            for (int v = v0; v < v1; v++) {
                const int8_t *T = lut8 + (size_t)v * 4 * 64;
                const uint8_t *ix = idx + (((size_t)rb * nv + v) * WO_BLK + ri) * 3;
                const unsigned b0 = ix[0], b1 = ix[1], b2 = ix[2];
                sum += T[b0 & 63] + T[64 + (((b0 >> 6) | (b1 << 2)) & 63)] +
                       T[128 + (((b1 >> 4) | (b2 << 4)) & 63)] + T[192 + ((b2 >> 2) & 63)];
            }
            const float p = lscale[v0 / 32] * (float)sum;
            acc = acc + p;
        }
        y[r] = acc * wo_f16(scale[r]);
    }
}

/* Dequantized expert matrix, fp32 [M][N]: recon = 0 + C0[i0] + C1[i1] +
 * C2[i2] per dimension, then times the row's fp16 scale — the order of the
 * reference's PyTorch oracle (tools/kimi_ref.py:262-270), with codebooks as
 * the engine decodes them (model.c:2916-2922, see wo_books_decode). */
void wo_vq_dequant(float *W, const uint8_t *idx, const uint16_t *scale,
                   const float *books, int M, int N, int cb_base)
{
    const int nv = N / WO_VEC;
    for (int r = 0; r < M; r++) {
        const int rb = r / WO_BLK, ri = r % WO_BLK;
        const float sc = wo_f16(scale[r]);
        for (int v = 0; v < nv; v++) {
            const uint8_t *ix = idx + (((size_t)rb * nv + v) * WO_BLK + ri) * WO_ST;
            for (int d = 0; d < WO_VEC; d++) {
                float t = 0.0f;
                for (int s = 0; s < WO_ST; s++)
                    t += books[((size_t)(cb_base + s) * WO_ENT + ix[s]) * WO_VEC + d];
                W[(size_t)r * N + v * WO_VEC + d] = t * sc;
            }
        }
    }
}

/* ---- trunk Q4G / Q8G --------------------------------------------------------- */

/* waste_mvq_rows_f32, portable branch (model.c:423-519): per group
 * part = sum_i w[i]*x[i] in i order (mul then add), acc += f16(ws[k])*part.
 * Q4: two nibbles per byte, low first, value = nibble - 8; Q8: int8.  Rows
 * at W + o*rowbytes, scales at ws + o*ng. */
void wo_mvq_rows(float *y, const void *Wv, const uint16_t *ws, const float *x,
                 int out, int in, int group, int bits, size_t rowbytes)
{
    const uint8_t *W = (const uint8_t *)Wv;
    const int ng = (in + group - 1) / group;
    for (int o = 0; o < out; o++) {
        const uint8_t *row = W + (size_t)o * rowbytes;
        float acc = 0.0f;
        for (int k = 0; k < ng; k++) {
            const int lim = (k * group + group <= in) ? group : in - k * group;
            float part = 0.0f;
            for (int i = 0; i < lim; i++) {
                const int gi = k * group + i;
                int q;
                if (bits == 4) {
                    const uint8_t b = row[gi >> 1];
                    q = (gi & 1) ? (b >> 4) - 8 : (b & 0x0f) - 8;
                } else {
                    q = (int8_t)row[gi];
                }
                const float p = (float)q * x[gi];
                part = part + p;
            }
            const float sp = wo_f16(ws[(size_t)o * ng + k]) * part;
            acc = acc + sp;
        }
        y[o] = acc;
    }
}

/* waste_deq_row (model.c:1137-1172) for `rows` rows. */
void wo_deq_rows(float *dst, const void *Wv, const uint16_t *ws, int rows,
                 int cols, int group, int bits, size_t rowbytes)
{
    const uint8_t *W = (const uint8_t *)Wv;
    const int ng = (cols + group - 1) / group;
    for (int r = 0; r < rows; r++) {
        const uint8_t *row = W + (size_t)r * rowbytes;
        for (int k = 0; k < ng; k++) {
            const float s = wo_f16(ws[(size_t)r * ng + k]);
            const int base = k * group;
            const int lim = (base + group <= cols) ? group : cols - base;
            for (int i = 0; i < lim; i++) {
                int v;
                if (bits == 8) v = (int8_t)row[base + i];
                else {
                    const uint8_t b = row[(base + i) >> 1];
                    v = (i & 1) ? (b >> 4) - 8 : (b & 0x0f) - 8;
                }
                dst[(size_t)r * cols + base + i] = s * (float)v;
            }
        }
    }
}

/* fp64 matvec over the dequantized rows: the tolerance reference for "the
 * reference's dequantised fp32 matvec" at any batch.  X is [batch][in],
 * Y is [batch][out]. */
void wo_deq_matmul_f64(double *Y, const void *W, const uint16_t *ws,
                       const float *X, int batch, int out, int in, int group,
                       int bits, size_t rowbytes)
{
    float *row = (float *)malloc((size_t)in * sizeof(float));
    for (int o = 0; o < out; o++) {
        wo_deq_rows(row, (const uint8_t *)W + (size_t)o * rowbytes,
                    ws + (size_t)o * ((in + group - 1) / group), 1, in, group,
                    bits, rowbytes);
        for (int b = 0; b < batch; b++) {
            double s = 0.0;
            const float *xb = X + (size_t)b * in;
            for (int i = 0; i < in; i++) s += (double)row[i] * (double)xb[i];
            Y[(size_t)b * out + o] = s;
        }
    }
    free(row);
}

/* quantize_q4g (convert.py:893-910): per group of `group` inputs,
 * scale = max|w| clamped to 1e-8, divided by 7; q = clamp(round(w/scale),
 * -8, 7) rounding half to even; stored nibble q+8, low nibble first;
 * scale stored fp16.  quantize_q8g (convert.py:913-925) is the same with
 * 127 and [-127, 127].  N must be a multiple of `group` (the configs'). */
void wo_quant_q(const float *W, int rows, int N, int group, int bits,
                uint8_t *q, uint16_t *scales)
{
    const int ng = N / group;
    const float div = bits == 4 ? 7.0f : 127.0f;
    const int lo = bits == 4 ? -8 : -127, hi = bits == 4 ? 7 : 127;
    for (int r = 0; r < rows; r++)
        for (int k = 0; k < ng; k++) {
            const float *g = W + (size_t)r * N + (size_t)k * group;
            float amax = 0.0f;
            for (int i = 0; i < group; i++) {
                const float a = fabsf(g[i]);
                if (a > amax) amax = a;
            }
            if (amax < 1e-8f) amax = 1e-8f;
            const float sc = amax / div;
            scales[(size_t)r * ng + k] = wo_f32_to_f16(sc);
            for (int i = 0; i < group; i++) {
                float t = rintf(g[i] / sc);
                int v = (int)t;
                if (v < lo) v = lo;
                if (v > hi) v = hi;
                const size_t gi = (size_t)r * N + (size_t)k * group + i;
                if (bits == 8) q[gi] = (uint8_t)(int8_t)v;
                else {
                    const uint8_t nib = (uint8_t)((v + 8) & 0x0f);
                    if (gi & 1) q[gi >> 1] = (uint8_t)(q[gi >> 1] | (nib << 4));
                    else q[gi >> 1] = nib;
                }
            }
        }
}

/* ---- RVQ encoder ----------------------------------------------------------- */

/* vq_step/vq_range (vq.c:50-96), scalar x86 branch: squared distance summed
 * over d in order with mul then add, strict `<` so the lowest index wins a
 * tie, the residual is v - C[best]; all stages in one pass. */
typedef struct {
    const float *X, *books;
    uint8_t *out;
    long b, e;
    int stages;
} wo_enc_job;

static void *wo_enc_range(void *p)
{
    const wo_enc_job *j = (const wo_enc_job *)p;
    float cur[WO_VEC], nxt[WO_VEC];
    for (long i = j->b; i < j->e; i++) {
        for (int d = 0; d < WO_VEC; d++) cur[d] = j->X[(size_t)i * WO_VEC + d];
        for (int s = 0; s < j->stages; s++) {
            const float *C = j->books + (size_t)s * WO_ENT * WO_VEC;
            int best = 0;
            float bestd = INFINITY;
            for (int c = 0; c < WO_ENT; c++) {
                float dd = 0.0f;
                for (int d = 0; d < WO_VEC; d++) {
                    const float t = cur[d] - C[c * WO_VEC + d];
                    const float tt = t * t;
                    dd = dd + tt;
                }
                if (dd < bestd) { bestd = dd; best = c; }
            }
            j->out[(size_t)i * j->stages + s] = (uint8_t)best;
            for (int d = 0; d < WO_VEC; d++) nxt[d] = cur[d] - C[best * WO_VEC + d];
            for (int d = 0; d < WO_VEC; d++) cur[d] = nxt[d];
        }
    }
    return NULL;
}

/* X [n][8] fp32, books [stages][256][8] fp32 -> out [n][stages]. */
void wo_vq_encode(const float *X, long n, const float *books, int stages,
                  uint8_t *out, int nthreads)
{
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 64) nthreads = 64;
    pthread_t th[64];
    int running[64] = {0};
    wo_enc_job jb[64];
    const long per = (n + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; t++) {
        jb[t].X = X; jb[t].books = books; jb[t].out = out; jb[t].stages = stages;
        jb[t].b = (long)t * per;
        jb[t].e = jb[t].b + per < n ? jb[t].b + per : n;
        if (jb[t].b >= jb[t].e) break;
        if (pthread_create(&th[t], NULL, wo_enc_range, &jb[t]) == 0) running[t] = 1;
        else wo_enc_range(&jb[t]);
    }
    for (int t = 0; t < nthreads; t++)
        if (running[t]) pthread_join(th[t], NULL);
}

/* block_indices (convert.py:777-792): codes [nvec][stages] for a row-major
 * [M][N] matrix (vector v of row r is entry r*N/8 + v) -> the blocked layout
 * [ceil(M/64)][N/8][64][stages], padding rows zero-filled. */
void wo_block_indices(const uint8_t *codes, int M, int N, int stages,
                      uint8_t *blocked)
{
    const int nv = N / WO_VEC, nb = (M + WO_BLK - 1) / WO_BLK;
    memset(blocked, 0, (size_t)nb * nv * WO_BLK * stages);
    for (int r = 0; r < M; r++)
        for (int v = 0; v < nv; v++)
            for (int s = 0; s < stages; s++)
                blocked[(((size_t)(r / WO_BLK) * nv + v) * WO_BLK + r % WO_BLK) * stages + s] =
                    codes[((size_t)r * nv + v) * stages + s];
}

/* quantize_vq (convert.py:821-851): per-row scale = max|w| clamped to 1e-8,
 * X = W/scale, encoded; the scale is stored fp16.  W [M][N] -> codes
 * [M*N/8][stages] (row-major vector order), scales [M]. */
void wo_quantize_vq(const float *W, int M, int N, const float *books,
                    uint8_t *codes, uint16_t *scales, int nthreads)
{
    float *X = (float *)malloc((size_t)M * N * sizeof(float));
    for (int r = 0; r < M; r++) {
        float amax = 0.0f;
        for (int i = 0; i < N; i++) {
            const float a = fabsf(W[(size_t)r * N + i]);
            if (a > amax) amax = a;
        }
        if (amax < 1e-8f) amax = 1e-8f;
        for (int i = 0; i < N; i++) X[(size_t)r * N + i] = W[(size_t)r * N + i] / amax;
        scales[r] = wo_f32_to_f16(amax);
    }
    wo_vq_encode(X, (long)M * N / WO_VEC, books, WO_ST, codes, nthreads);
    free(X);
}

/* ---- router and activation --------------------------------------------------- */

/* waste_qwen_moe_route (qwen_moe.c:10-44): softmax over E in fp32 (max
 * subtracted, sequential sum, z floored at 1e-20), then K passes selecting
 * the strictly greatest unused probability (lowest id wins ties), weights in
 * selection order, optional renormalization by their sequential sum. */
int wo_qwen_route(const float *logits, int E, int K, int renorm, int *idx,
                  float *w)
{
    for (int j = 0; j < K; j++) { idx[j] = 0; w[j] = 0.0f; }
    if (!logits || E < 1 || K < 1 || K > E) return -1;
    float *prob = (float *)malloc((size_t)E * sizeof(float));
    uint8_t *used = (uint8_t *)calloc((size_t)E, 1);
    float m = logits[0];
    for (int e = 1; e < E; e++) if (logits[e] > m) m = logits[e];
    float z = 0.0f;
    for (int e = 0; e < E; e++) { prob[e] = expf(logits[e] - m); z += prob[e]; }
    if (z < 1e-20f) z = 1e-20f;
    for (int e = 0; e < E; e++) prob[e] /= z;
    for (int j = 0; j < K; j++) {
        int best = -1;
        float bv = -1.0f;
        for (int e = 0; e < E; e++) {
            if (used[e]) continue;
            if (prob[e] > bv) { bv = prob[e]; best = e; }
        }
        idx[j] = best >= 0 ? best : 0;
        w[j] = best >= 0 ? prob[best] : 0.0f;
        if (best >= 0) used[best] = 1;
    }
    if (renorm && K > 1) {
        float s = 0.0f;
        for (int j = 0; j < K; j++) s += w[j];
        if (s > 1e-20f)
            for (int j = 0; j < K; j++) w[j] /= s;
    }
    free(prob);
    free(used);
    return 0;
}

/* moe_layer's router (model.c:5466-5556), the Kimi / GLM / DeepSeek path:
 *   scores (router_scores, model.c:5466-5486), func as the engine numbers
 *   them (model.h:179-181): 0 sigmoid 1 / (1 + expf(-x)); 1 softmax (max
 *   from -1e30, expf(l - max), sum in e order, each divided by the sum);
 *   2 sqrt(softplus(x)), softplus = x above 30, else log1pf(expf(x));
 *   selection (model.c:5524-5545): K passes, value score + bias (bias NULL
 *   = 0; the bias moves the ranking only), strict > from -1e30, the first
 *   (lowest) id on ties, skipping ids already taken; w[j] = score[idx[j]];
 *   renorm (K > 1): w[j] /= (sum_j w + 1e-20), the sum in j order
 *   (model.c:5547-5551); then w[j] *= routed_scale (model.c:5552).
 * score_out (optional, [E]) receives the scores. */
int wo_route_scored(const float *logit, int E, int K, int func, const float *bias,
                    int renorm, float routed_scale, int *idx, float *w, float *score_out)
{
    for (int j = 0; j < K; j++) { idx[j] = 0; w[j] = 0.0f; }
    if (!logit || E < 1 || K < 1 || K > E || K > 64) return -1;
    float *score = (float *)malloc((size_t)E * sizeof(float));
    if (func == 2) {
        for (int e = 0; e < E; e++) {
            const float x = logit[e];
            const float sp = x > 30.0f ? x : log1pf(expf(x));
            score[e] = sqrtf(sp);
        }
    } else if (func == 1) {
        float mx = -1e30f;
        for (int e = 0; e < E; e++) if (logit[e] > mx) mx = logit[e];
        float sum = 0.0f;
        for (int e = 0; e < E; e++) { score[e] = expf(logit[e] - mx); sum += score[e]; }
        for (int e = 0; e < E; e++) score[e] /= sum;
    } else {
        for (int e = 0; e < E; e++) score[e] = 1.0f / (1.0f + expf(-logit[e]));
    }
    for (int j = 0; j < K; j++) {
        int best = -1;
        float bv = -1e30f;
        for (int e = 0; e < E; e++) {
            int taken = 0;
            for (int q = 0; q < j; q++) if (idx[q] == e) { taken = 1; break; }
            if (taken) continue;
            const float v = score[e] + (bias ? bias[e] : 0.0f);
            if (v > bv) { bv = v; best = e; }
        }
        idx[j] = best;
        w[j] = best >= 0 ? score[best] : 0.0f;
    }
    if (renorm && K > 1) {
        float sm = 0.0f;
        for (int j = 0; j < K; j++) sm += w[j];
        for (int j = 0; j < K; j++) w[j] /= (sm + 1e-20f);
    }
    for (int j = 0; j < K; j++) w[j] *= routed_scale;
    if (score_out) memcpy(score_out, score, (size_t)E * sizeof(float));
    free(score);
    for (int j = 0; j < K; j++) if (idx[j] < 0) return -2;
    return 0;
}

/* SwiGLU (model.c:1231, 1264): g = silu(g) * u, silu(v) = v / (1 + expf(-v)). */
void wo_swiglu(float *g, const float *u, int n)
{
    for (int i = 0; i < n; i++) {
        const float v = g[i];
        g[i] = (v / (1.0f + expf(-v))) * u[i];
    }
}

/* ---- one MoE layer ------------------------------------------------------------ */

/* The expert FFN of one token, composed the way qwen_moe_layer
 * (model.c:8180-8405) and moe_layer (model.c:5488-5940) compose it:
 *   logits = Wr . x (fp32, sequential dot), route (wo_qwen_route);
 *   gate/up LUTs once from x (codebooks cb+0, cb+3); per routed expert j:
 *   g = vq_rows(gate), u = vq_rows(up), h = silu(g)*u, down LUT from h
 *   (cb+6), acc_j = vq_rows(down);
 *   out = sum_j w[j]*acc_j in route order (model.c:8385-8400), starting 0;
 *   shared expert (ffn, model.c:5391): a = Wsg.x, b = Wsu.x, h = silu(a)*b,
 *   s = Wsd.h through wo_mvq_rows; out += sg * s with sg = sigmoid(wsgate.x)
 *   when a shared gate is given (model.c:8155-8181, 8402), else 1
 *   (model.c:5932-5939).
 * recs[e] points at expert e's WEXP record (48-byte header; gate/up/down
 * index offsets and the scale offset read from it, waste_format.h:98-130).
 * Results: out [hid]; optional idx/w [K]; optional acc [K][hid]. */
typedef struct {
    uint32_t magic;
    uint16_t layer, expert_id;
    uint8_t fmt, flags;
    uint16_t codebook_id, lowrank_id, reserved0;
    uint32_t rec_4k_blocks, gate_off, up_off, down_off, chan_corr_off, crc32;
    uint32_t reserved1[2];
} wo_hdr;

void wo_expert_ffn(const uint8_t *rec, const float *booksT, const float *lut_g,
                   const float *lut_u, int hid, int inter, float *acc)
{
    const wo_hdr *h = (const wo_hdr *)rec;
    const uint16_t *sc = (const uint16_t *)(rec + h->chan_corr_off);
    float *g = (float *)malloc((size_t)inter * sizeof(float));
    float *u = (float *)malloc((size_t)inter * sizeof(float));
    float *lut_d = (float *)malloc((size_t)(inter / WO_VEC) * WO_ST * WO_ENT * sizeof(float));
    wo_vq_rows(g, rec + h->gate_off, sc, lut_g, inter, hid / WO_VEC);
    wo_vq_rows(u, rec + h->up_off, sc + inter, lut_u, inter, hid / WO_VEC);
    wo_swiglu(g, u, inter);
    wo_lut_build(lut_d, booksT, g, inter / WO_VEC, h->codebook_id + 2 * WO_ST);
    wo_vq_rows(acc, rec + h->down_off, sc + 2 * inter, lut_d, hid, inter / WO_VEC);
    free(g); free(u); free(lut_d);
}

/* The router logits of wo_moe_layer for T tokens at once: logits[t][e] =
 * sum_i Wr[e][i] * x[t][i], fp32, i ascending (the router matvec of
 * qwen_moe_layer, model.c:8180-8405, as the engine's scalar matvec sums it).
 * Lets a test check the routing of many tokens without running each one's
 * experts. */
void wo_router_logits(const float *x, int T, int hid, const float *Wr, int E, float *logits)
{
    for (int t = 0; t < T; t++)
        for (int e = 0; e < E; e++) {
            float s = 0.0f;
            for (int i = 0; i < hid; i++) s += Wr[(size_t)e * hid + i] * x[(size_t)t * hid + i];
            logits[(size_t)t * E + e] = s;
        }
}

/* The router a layer uses: kind 0 wo_qwen_route, kind 1 wo_route_scored. */
static int wo_route_kind = 0, wo_route_func = 0;
static const float *wo_route_bias = NULL;
static float wo_route_scale = 1.0f;

void wo_set_router(int kind, int func, const float *bias, float routed_scale)
{
    wo_route_kind = kind;
    wo_route_func = func;
    wo_route_bias = bias;
    wo_route_scale = routed_scale;
}

int wo_moe_layer(const float *x, int hid, int inter, int E, int K, int renorm,
                 const float *Wr, const uint8_t *const *recs,
                 const float *booksT,
                 const void *Wsg, const uint16_t *ssg, const void *Wsu,
                 const uint16_t *ssu, const void *Wsd, const uint16_t *ssd,
                 int sgroup, int sbits, int shared_inter,
                 const float *wsgate,
                 float *out, int *idx_out, float *w_out, float *acc_out)
{
    float *logits = (float *)malloc((size_t)E * sizeof(float));
    for (int e = 0; e < E; e++) {
        float s = 0.0f;
        for (int i = 0; i < hid; i++) s += Wr[(size_t)e * hid + i] * x[i];
        logits[e] = s;
    }
    int idx[64];
    float w[64];
    if (K > 64 || (wo_route_kind == 1
                       ? wo_route_scored(logits, E, K, wo_route_func, wo_route_bias, renorm,
                                         wo_route_scale, idx, w, NULL)
                       : wo_qwen_route(logits, E, K, renorm, idx, w)) != 0) {
        free(logits);
        return -1;
    }
    free(logits);
    const int nv = hid / WO_VEC;
    const wo_hdr *h0 = (const wo_hdr *)recs[idx[0]];
    float *lut_g = (float *)malloc((size_t)nv * WO_ST * WO_ENT * sizeof(float));
    float *lut_u = (float *)malloc((size_t)nv * WO_ST * WO_ENT * sizeof(float));
    wo_lut_build(lut_g, booksT, x, nv, h0->codebook_id + 0);
    wo_lut_build(lut_u, booksT, x, nv, h0->codebook_id + WO_ST);
    float *acc = (float *)malloc((size_t)K * hid * sizeof(float));
    for (int j = 0; j < K; j++)
        wo_expert_ffn(recs[idx[j]], booksT, lut_g, lut_u, hid, inter,
                      acc + (size_t)j * hid);
    for (int i = 0; i < hid; i++) out[i] = 0.0f;
    for (int j = 0; j < K; j++)
        for (int i = 0; i < hid; i++) {
            const float p = w[j] * acc[(size_t)j * hid + i];
            out[i] = out[i] + p;
        }
    if (Wsg) {
        const int sn = shared_inter;
        const size_t rb_h = (size_t)((hid + sgroup - 1) / sgroup) * sgroup * sbits / 8;
        const size_t rb_i = (size_t)((sn + sgroup - 1) / sgroup) * sgroup * sbits / 8;
        float *a = (float *)malloc((size_t)sn * sizeof(float));
        float *b = (float *)malloc((size_t)sn * sizeof(float));
        float *s = (float *)malloc((size_t)hid * sizeof(float));
        wo_mvq_rows(a, Wsg, ssg, x, sn, hid, sgroup, sbits, rb_h);
        wo_mvq_rows(b, Wsu, ssu, x, sn, hid, sgroup, sbits, rb_h);
        wo_swiglu(a, b, sn);
        wo_mvq_rows(s, Wsd, ssd, a, hid, sn, sgroup, sbits, rb_i);
        float sg = 1.0f;
        if (wsgate) {
            float t = 0.0f;
            for (int i = 0; i < hid; i++) t += wsgate[i] * x[i];
            sg = 1.0f / (1.0f + expf(-t));
        }
        for (int i = 0; i < hid; i++) {
            const float p = sg * s[i];
            out[i] = out[i] + p;
        }
        free(a); free(b); free(s);
    }
    if (idx_out) for (int j = 0; j < K; j++) idx_out[j] = idx[j];
    if (w_out) for (int j = 0; j < K; j++) w_out[j] = w[j];
    if (acc_out) memcpy(acc_out, acc, (size_t)K * hid * sizeof(float));
    free(acc); free(lut_g); free(lut_u);
    return 0;
}
