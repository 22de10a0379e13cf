/*
 * ref_shim.c — TEST INFRASTRUCTURE ONLY.  The reference engine's own code,
 * reached from Python so that the oracle restatement (warp_oracle.c) and
 * the golden fixtures can be checked against it.
 *
 * This translation unit #includes the reference's src/model.c, so the
 * static kernels the expert FFN is made of (vq_rows, vq_build_lut,
 * experts_staged, moe_expert_range, ffn, matvec_t) are callable unchanged.
 * It is compiled by oracle/Makefile straight from the reference sources into
 * oracle/_ref/ and linked with the reference's other objects.  Nothing in
 * the product links or loads it: only tests/, the golden-fixture script and
 * bench.py's reference arm do, and only as a checker or the timed CPU
 * baseline.
 *
 * Every entry point below is a thin argument adapter around one reference
 * function; the file:line it reaches is named beside it.
 */
#include "model.c"

/* ---- set-up ------------------------------------------------------------ */

/* waste_backend_init (backend.c:169) fills waste_k with the portable kernels
 * and then the AVX-512/AVX2 ones this CPU supports.  The pool size is the
 * caller's: 1 for a scalar comparison, 0 for every core (the CPU baseline). */
int ref_init(int nthreads)
{
    prof_on = 0;
    waste_backend_init(WASTE_BE_AUTO);
    waste_pool_init(nthreads, NULL);
    return waste_pool_threads();
}

const char *ref_backend_name(void) { return waste_backend_name(); }

/* ---- trunk dequant-matvec (model.c:423 / simd_avx512.c:20) -------------- */

/* slot 0: the dispatched kernel (waste_k.mvq_rows_f32, AVX-512 here);
 * slot 1: the portable waste_mvq_rows_f32.  Rows are split over the pool the
 * way run_rows (model.c:805) splits them. */
void ref_mvq_rows(float *y, const void *W, const uint16_t *ws, const float *x,
                  int out, int in, int group, int bits, size_t rowbytes,
                  int slot)
{
    const int ng = (in + group - 1) / group;
    mvq_arg a = { y, (const int8_t *)W, ws, NULL, x, in, ng, group, bits,
                  rowbytes };
    waste_range_fn fn = slot == 1 ? waste_mvq_rows_f32 : waste_k.mvq_rows_f32;
    waste_parallel_for_work(out, mv_chunk(out, rowbytes), fn, &a,
                            (size_t)out * rowbytes);
}

/* waste_deq_row (model.c:1137): one trunk row dequantized to fp32. */
void ref_deq_rows(float *dst, const void *W, const uint16_t *ws, int rows,
                  int cols, int group, int bits, size_t rowbytes)
{
    waste_tensor t;
    memset(&t, 0, sizeof t);
    t.q = (int8_t *)W;
    t.qs = (uint16_t *)ws;
    t.group = group;
    t.bits = bits;
    t.rowbytes = rowbytes;
    for (int r = 0; r < rows; r++)
        waste_deq_row(&t, r, cols, dst + (size_t)r * cols);
}

/* ---- VQ3R --------------------------------------------------------------- */

/* Codebook decode exactly as the loader does it (model.c:2911-2945): fp16
 * with subnormals flushed to zero, then the [book][dim][entry] transpose. */
void ref_books_from_f16(const uint16_t *h, int n_books, int entries,
                        int vec_dim, float *books, float *booksT)
{
    const size_t per = (size_t)entries * vec_dim;
    for (size_t i = 0; i < (size_t)n_books * per; i++) {
        const uint16_t v = h[i];
        const uint32_t sign = (uint32_t)(v >> 15) << 31;
        uint32_t e = (v >> 10) & 0x1f, man = v & 0x3ff, bits;
        bits = e ? (sign | ((e + 112u) << 23) | (man << 13)) : sign;
        memcpy(&books[i], &bits, 4);
    }
    for (int b = 0; b < n_books; b++)
        for (int c = 0; c < entries; c++)
            for (int d = 0; d < vec_dim; d++)
                booksT[(size_t)b * per + (size_t)d * entries + c] =
                    books[(size_t)b * per + (size_t)c * vec_dim + d];
}

/* LUT build.  slot 0: waste_k.lutb_range (lutb_range_avx512 here,
 * simd_avx512.c:90), slot 1: the portable waste_lutb_range (model.c:3815). */
void ref_lutb(float *lut, const float *booksT, const float *x, int nv,
              int cb_base, int stages, int entries, int vec_dim, int slot)
{
    lutb_arg a = { lut, booksT, x, cb_base, stages, entries, vec_dim };
    (slot == 1 ? waste_lutb_range : waste_k.lutb_range)(0, nv, &a);
}

/* VQ4P: vq_quant_lut (model.c:4063) and the apply, slot 0 the dispatched
 * waste_k.vq_rows_p6 (vq_rows_p6_avx512 here, simd_avx512.c:129), slot 1
 * the portable waste_vq_rows_p6 (model.c:4076). */
void ref_vq_quant_lut(const float *lut, int nv, int st, int en, int8_t *q, float *scale)
{
    vq_quant_lut(lut, nv, st, en, q, scale);
}

void ref_vq_rows_p6(float *y, const uint8_t *idx, const uint16_t *scale, const int8_t *lut8,
                    const float *lscale, int M, int nv, int slot)
{
    vqp_arg a = { y, idx, scale, lut8, lscale, nv };
    (slot == 1 ? waste_vq_rows_p6 : waste_k.vq_rows_p6)(0, M, &a);
}

/* vq_rows (model.c:3909) over all M rows, serially. */
void ref_vq_rows(float *y, const uint8_t *idx, const uint16_t *scale,
                 const float *lut, int M, int nv, int stages, int entries)
{
    vq_arg a = { y, idx, scale, lut, nv, stages, entries };
    vq_rows(0, M, &a);
}

/* waste_vq_encode (vq.c:99) is exported by vq.c itself. */

/* ---- routing and activation ---------------------------------------------- */

int ref_qwen_route(const float *logits, int E, int K, int renorm, int *idx,
                   float *w)
{
    float *prob = (float *)malloc((size_t)E * sizeof(float));
    uint8_t *used = (uint8_t *)malloc((size_t)E);
    const int rc = waste_qwen_moe_route(logits, E, K, renorm, idx, w, prob, used);
    free(prob);
    free(used);
    return rc;
}

/* router_scores (model.c:5466-5486) for one token: score[e] from logit[e]
 * with the engine's score function (model.h:179-181). */
void ref_router_scores(int score_func, const float *logit, float *score, int E)
{
    waste_config c;
    memset(&c, 0, sizeof c);
    c.score_func = score_func;
    router_scores(&c, logit, score, E);
}

/* waste_act_pair_range (model.c:1251) with the plain SwiGLU config. */
void ref_swiglu(float *g, const float *u, int n)
{
    waste_config c;
    memset(&c, 0, sizeof c);
    waste_act_pair_range(&c, g, u, n);
}

/* ---- the MoE layer ------------------------------------------------------- *
 *
 * A minimal waste_model carrying only what the expert path reads: the
 * transposed codebooks, the VQ geometry and the per-expert scratch of the
 * expert-parallel path.  Records are whole WEXP records (48-byte header
 * first), exactly what the expert cache hands moe_layer. */

typedef struct {
    waste_model *m;
    int hid, inter, K;
} ref_moe;

void *ref_moe_new(const float *booksT, int n_books, int hid, int inter, int K)
{
    ref_moe *r = (ref_moe *)calloc(1, sizeof *r);
    waste_model *m = (waste_model *)calloc(1, sizeof *m);
    if (!r || !m) { free(r); free(m); return NULL; }
    m->codebooksT = (float *)booksT;
    m->n_books = n_books;
    m->vec_dim = 8;
    m->cb_entries = 256;
    m->stages = 3;
    m->index_bits = 8;
    const int big = hid > inter ? hid : inter;
    m->xlut_sz = (size_t)(inter / 8) * 3 * 256;
    m->xga = (float *)calloc((size_t)K * inter, sizeof(float));
    m->xub = (float *)calloc((size_t)K * inter, sizeof(float));
    m->xacc = (float *)calloc((size_t)K * hid, sizeof(float));
    m->xlut = (float *)calloc((size_t)K * m->xlut_sz, sizeof(float));
    m->lut = (float *)calloc((size_t)3 * (big / 8) * 3 * 256, sizeof(float));
    m->ff = (float *)calloc((size_t)2 * big, sizeof(float));
    m->h = (float *)calloc((size_t)big, sizeof(float));
    m->e_gate = (float *)calloc((size_t)big, sizeof(float));
    r->m = m; r->hid = hid; r->inter = inter; r->K = K;
    return r;
}

void ref_moe_free(void *p)
{
    ref_moe *r = (ref_moe *)p;
    if (!r) return;
    waste_model *m = r->m;
    free(m->xga); free(m->xub); free(m->xacc); free(m->xlut);
    free(m->lut); free(m->ff); free(m->h); free(m->e_gate);
    free(m);
    free(r);
}

/* K routed experts for one token, through experts_staged (model.c:4330, the
 * path qwen_moe_layer takes for resident experts, model.c:8266-8300) or
 * through moe_expert_range (model.c:4208, the expert-parallel path) when
 * `per_expert` is set.  Leaves each expert's unweighted down output in
 * acc[j*hid ...], and writes out[] = sum_j w[j]*acc_j in route order
 * (model.c:8385-8400). */
void ref_moe_experts(void *p, const uint8_t *const *recs, const float *w,
                     const float *x, float *acc, float *out, int per_expert)
{
    ref_moe *r = (ref_moe *)p;
    waste_model *m = r->m;
    const int hid = r->hid, inter = r->inter, K = r->K;
    const int lut_sz = (hid / 8) * 3 * 256;
    float *lut_gate = m->lut, *lut_up = lut_gate + lut_sz;
    const waste_expert_hdr *h0 = (const waste_expert_hdr *)recs[0];
    vq_build_lut(m, lut_gate, h0->codebook_id + 0, x, hid, 3, 256, 8, NULL, NULL);
    vq_build_lut(m, lut_up, h0->codebook_id + 3, x, hid, 3, 256, 8, NULL, NULL);
    int list[64];
    for (int j = 0; j < K; j++) list[j] = j;
    if (per_expert) {
        xpar_arg pa = { m, &m->cfg, (const uint8_t **)recs, w, 0, inter, hid,
                        lut_gate, lut_up, NULL, NULL, NULL, NULL, NULL };
        waste_parallel_for(K, 1, moe_expert_range, &pa);
    } else {
        experts_staged(m, (const uint8_t **)recs, list, K, inter, hid,
                       lut_gate, lut_up);
    }
    memset(out, 0, (size_t)hid * sizeof(float));
    for (int j = 0; j < K; j++) {
        const float *accj = m->xacc + (size_t)j * hid;
        const float wj = w[j];
        for (int i = 0; i < hid; i++) out[i] += wj * accj[i];
    }
    if (acc) memcpy(acc, m->xacc, (size_t)K * hid * sizeof(float));
}

/* The shared expert through ffn (model.c:5391): three trunk matvecs through
 * matvec_t -> run_rows(waste_k.mvq_rows_f32) and the SwiGLU between them.
 * Q4G/Q8G payloads in the trunk layout: row o at W + o*rowbytes, one fp16
 * scale per group. */
void ref_shared_expert(void *p, const void *Wg, const uint16_t *sg,
                       const void *Wu, const uint16_t *su,
                       const void *Wd, const uint16_t *sd,
                       int group, int bits, const float *x, float *y)
{
    ref_moe *r = (ref_moe *)p;
    waste_model *m = r->m;
    const int hid = r->hid, inter = r->inter;
    waste_tensor t[3];
    memset(t, 0, sizeof t);
    const void *W[3] = { Wg, Wu, Wd };
    const uint16_t *S[3] = { sg, su, sd };
    const int in[3] = { hid, hid, inter };
    for (int i = 0; i < 3; i++) {
        const int ng = (in[i] + group - 1) / group;
        t[i].q = (int8_t *)W[i];
        t[i].qs = (uint16_t *)S[i];
        t[i].group = group;
        t[i].bits = bits;
        t[i].rowbytes = (size_t)ng * group * bits / 8;
        snprintf(t[i].name, sizeof t[i].name, "shared.%d", i);
    }
    ffn(m, &t[0], &t[1], &t[2], x, y, inter, hid, 1.0f, 0);
}

/* The router's logits through the reference's fp32 matvec (matvec,
 * model.c:791-797: mv_rows split over the pool by 64-row chunks). */
void ref_matvec_f32(float *y, const float *W, const float *x, int out, int in)
{
    matvec(y, W, x, out, in);
}

/* Pool size actually in use (the baseline reports it). */
int ref_threads(void) { return waste_pool_threads(); }
