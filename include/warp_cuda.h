/*
 * warp_cuda.h — the C ABI of libwarp_cuda.so, the B200 (sm_100a) backend for
 * WARP's quantized expert FFN.
 *
 * Two layers of entry points:
 *
 *  1. The drop-in boundary the reference engine binds (waste_backend.h's
 *     plugin table).  These take HOST pointers, exactly as the CPU kernels
 *     they replace do, and keep device mirrors of the weights they are given.
 *       - waste_register_cuda     replaces the declaration the reference
 *                                 already makes at src/backend.c:58 and calls
 *                                 at src/backend.c:209.
 *       - waste_cuda_vq3r         the batch VQ3R apply with the job ABI of
 *                                 src/waste_metal.h:31-44 (waste_metal_vq3r).
 *       - waste_cuda_release_host_buffers  the hook of
 *                                 src/backend.c:229-235.
 *
 *  2. Device-resident entry points (device pointers, an explicit stream) that
 *     the repository's own MoE driver, tests and benchmark use.  Each names
 *     the reference function whose arithmetic it computes.
 *
 * Every function returns 0 (WARP_OK) or a negative warp_status; the message
 * of the last failure on the calling thread is warp_last_error().  No entry
 * point exits or falls back to the CPU: a failure is returned.  None prints
 * except waste_metal_selftest, a diagnostic whose contract is to print.
 */
#ifndef WARP_CUDA_H
#define WARP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WARP_API __attribute__((visibility("default")))
#else
#define WARP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    WARP_OK = 0,
    WARP_E_ARG = -1,      /* a size, pointer or alignment the kernel cannot take */
    WARP_E_CUDA = -2,     /* a CUDA runtime error (message in warp_last_error)   */
    WARP_E_NODEV = -3,    /* no usable sm_100 device                             */
    WARP_E_NOMEM = -4,    /* device allocation failed                            */
    WARP_E_TIMEOUT = -5,  /* a bounded device wait gave up                       */
    WARP_E_FORMAT = -6,   /* an expert record or codebook that does not parse    */
} warp_status;

/* ---- library ---------------------------------------------------------------- */

WARP_API const char *warp_version(void);            /* "warp_b200 <ver> sm_100a"       */
WARP_API const char *warp_last_error(void);         /* thread-local, never NULL        */
/* 1 when device `dev` is an sm_100 part this build can run on, else 0. */
WARP_API int warp_device_ok(int dev);
/* Kernels launched by this library since load (all entry points, all
 * streams); the benchmark reads it to count its own launches. */
WARP_API uint64_t warp_launch_count(void);

/* ---- 1. reference plugin boundary (host pointers) --------------------------- */

/* Opaque here; the engine passes its waste_kernels table (waste_backend.h:69).
 * Fills mvq_rows_f32 with the device matvec, sets on_device = 1 and
 * device_min_bytes, and returns "CUDA sm_100a", or NULL to decline (no
 * device, init failure, WARP_CUDA_DISABLE set).  Idempotent. */
WARP_API const char *waste_register_cuda(void *waste_kernels_table);

/* The job of src/waste_metal.h:31-40, field for field. */
typedef struct {
    float         *y;
    const uint8_t *rec;
    size_t         rec_bytes;
    uint32_t       idx_off, sc_off;
    const float   *lut;
    size_t         lut_bytes;
    uint32_t       lut_off;
    int            m, nv, stages, entries;
} warp_vq_job;

/* waste_metal_vq3r (src/waste_metal.h:42-44): y = scale * sum_v T0+T1+T2 for
 * every job, on the device.  0 if every job ran; non-zero and nothing
 * written otherwise (the caller then computes them itself). */
WARP_API int waste_cuda_vq3r(const warp_vq_job *jobs, int n);

/* Drop every device mirror keyed by a host pointer (backend.c:229-235). */
WARP_API void waste_cuda_release_host_buffers(void);

/* How many slot calls ran the engine's CPU kernel instead of the device
 * (a shape the device matvec does not take, or a device failure). */
WARP_API unsigned long long warp_cuda_fallback_count(void);

/* The boundary's counters: out[0] mvq_rows_f32 slot calls run on the
 * device, out[1] slot calls handed to the engine's CPU kernel, out[2] batch
 * VQ3R calls run, out[3] jobs in them.  With WARP_CUDA_STATS=<path> set in
 * the environment at registration, the same four are appended to <path> as
 * one JSON line at process exit. */
WARP_API int warp_cuda_stats(unsigned long long *out);

/* The engine's Metal hooks, answered by CUDA, so that the reference builds
 * with -DWASTE_ENABLE_CUDA=1 -DWASTE_ENABLE_METAL=1 against this library
 * with model.c and backend.c unchanged:
 *   waste_metal_vq3r      src/waste_metal.h:42-44, called by moe_layer
 *                         (src/model.c:5665-5792) when WASTE_METAL_MOE=1;
 *                         the same as waste_cuda_vq3r.
 *   waste_register_metal  src/backend.c:55, 211-213; declines (NULL): the
 *                         CUDA registration, which backend.c runs first,
 *                         already filled the table.
 *   waste_metal_release_host_buffers  src/backend.c:229-235; the same as
 *                         waste_cuda_release_host_buffers. */
WARP_API int waste_metal_vq3r(const warp_vq_job *jobs, int n);
WARP_API const char *waste_register_metal(void *waste_kernels_table);
WARP_API void waste_metal_release_host_buffers(void);
/* waste_metal_selftest (src/metal.m:403-460, called by tests/test_forward.c
 * :271-275 when WASTE_METAL_SELFTEST is set): the one entry point that
 * prints, because printing is its contract.  It times the device Q4 trunk
 * matvec (M 12288, K 7168, group 128; weights reused, rotated over 32
 * copies, and rotated with the x / y host copies) and writes one line per
 * mode to stderr.  Does nothing before waste_register_cuda succeeded. */
WARP_API void waste_metal_selftest(void);

/* ---- 2. device-resident kernels ---------------------------------------------- */

/* Trunk / shared-expert dequant-matvec, the arithmetic of waste_mvq_rows_f32
 * (src/model.c:423-519): Y[b][o] = sum_k f16(ws[o*ng+k]) *
 * sum_i q(o, k*group+i) * X[b][k*group+i].  bits 4 (two nibbles per byte,
 * low first, value nibble-8) or 8 (int8).  X is fp32 (x_bf16 = 0) or bf16
 * (x_bf16 = 1), [batch][in]; Y fp32 [batch][out].  W rows at W + o*rowbytes;
 * rowbytes and W must be 16-byte aligned, in a multiple of 32 (bits 4) or
 * 16 (bits 8), group a multiple of 32, batch 1..64 (the engine's prefill
 * chunk, WASTE_CHUNK_MAX src/model.h:532; waste_matmul_t / mmq_rows,
 * src/model.c:6964-7028, for batch >= 2).  Batch >= 2 runs on the tensor
 * cores with a fragment scratch the library keeps per (device, stream),
 * allocated on the first call that needs it (or a larger one), so make that
 * call before capturing the stream into a CUDA graph. */
WARP_API int warp_mvq_matvec(const void *W, const uint16_t *ws, const void *X,
                    int x_bf16, float *Y, int batch, int out, int in,
                    int group, int bits, size_t rowbytes, void *stream);

/* The tensor-core matmul's bounded waits (batch >= 2): WARP_OK, or
 * WARP_E_TIMEOUT if a wait gave up since the last clear (that launch's
 * output is incomplete).  Synchronises the device; clear = 1 resets. */
WARP_API int warp_mvq_status(int clear);

/* VQ3R table build, the arithmetic of lutb_range_avx512
 * (src/simd_avx512.c:90-127): lut[v][s][c] = FMA chain over d = 0..7 from 0
 * of x[8v+d] * booksT[cb_base+s][d][c].  booksT is [n_books][8][256] fp32
 * (the engine's codebooksT, src/model.c:2929-2941).  Bit-exact. */
WARP_API int warp_vq_lut_build(float *lut, const float *booksT, const float *x,
                      int nv, int cb_base, void *stream);

/* VQ3R apply, vq_rows (src/model.c:3909-3977): y[r] = f16(scale[r]) *
 * sum_v ((T0[i0] + T1[i1]) + T2[i2]) over the blocked index layout
 * [ceil(M/64)][nv][64][3].  ordered = 1 sums v ascending exactly as vq_rows
 * does (bit-exact); ordered = 0 is the bandwidth kernel (fp32, tolerance). */
WARP_API int warp_vq_apply(float *y, const uint8_t *idx, const uint16_t *scale,
                  const float *lut, int M, int nv, int ordered, void *stream);

/* warp_vq_apply's bandwidth path (ordered = 0) without any device
 * allocation.  No counterpart in the reference: it exists for callers that
 * must not touch a device allocator at all — an engine that sizes all of HBM
 * once at load and must not grow mid-step, a context whose stream-ordered
 * memory pool is unsupported or disabled, a decode loop that must not take an
 * allocator lock while a step runs.  Its scratch is a fixed 8 MiB of
 * module-scope device memory per device: the call returns WARP_E_ARG with a
 * message when ceil(nv/32) * 98304 + ceil(ceil(nv/32) * M * 4 / 256) * 256 +
 * 256 bytes exceed that (M <= 8192 with nv <= 896 fits).  The first call on
 * a device looks up the scratch's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.
 * Calls that overlap on one device (other streams or host threads) share the
 * scratch and race: serialise them.  Synchronises `stream` before returning,
 * like warp_vq_apply. */
WARP_API int warp_vq_apply_noalloc(float *y, const uint8_t *idx, const uint16_t *scale,
                          const float *lut, int M, int nv, void *stream);

/* The VQ4P format (FORMAT.md "VQ4P record"): four residual stages of 64
 * entries, the four 6-bit indices of a (row, vector position) packed into
 * three bytes, applied through an int8 table.
 *   warp_vq4p_lut: the table of x and its int8 quantisation, vq_build_lut
 *   with 4 stages of 64 entries (lutb_range, src/model.c:3815-3852, the FMA
 *   chain over d from 0) then vq_quant_lut (src/model.c:3996-4068): q
 *   [nv][4][64] int8 and lscale [ceil(nv/32)], one scale per 32 positions.
 *   booksT is [n_books][8][64] fp32; books cb_base..cb_base+3 are used.
 *   warp_vq4p_apply: waste_vq_rows_p6 (src/model.c:4076-4113): idx in the
 *   blocked layout [ceil(M/64)][nv][64][3 bytes]; per block of 32 positions
 *   the integer sum of the four lookups, acc += lscale[blk] * sum in block
 *   order, y = acc * f16(scale[r]).
 * Both bit-exact against the reference's portable kernels. */
WARP_API int warp_vq4p_lut(int8_t *q, float *lscale, const float *booksT, int n_books,
                  const float *x, int nv, int cb_base, void *stream);
WARP_API int warp_vq4p_apply(float *y, const uint8_t *idx, const uint16_t *scale,
                    const int8_t *lut8, const float *lscale, int M, int nv, void *stream);

/* VQ3R dequant GEMM for T tokens at once — the prefill form of vq_rows
 * (src/model.c:3909-3977; moe_chunk, src/model.c:7110-7290, applies it per
 * token):  Y[t][r] = f16(scale[r]) * sum_k W~[r][k] * X[t][k], where
 * W~[r][8v+d] = (C0[i0][d] + C1[i1][d]) + C2[i2][d] is formed in fp32 and
 * rounded once to fp16, X is rounded to fp16, and products accumulate in
 * fp32 on the tensor cores (tcgen05).  idx is the blocked index layout of an
 * M x N matrix, books [n_books][256][8] fp32 from cb_base, X [T][N] and
 * Y [T][M] fp32.  Agrees with the fp32 reference to the FFN tolerance
 * (2e-3 relative L2); not bit-exact.  No host synchronisation. */
WARP_API int warp_vq_matmul(float *Y, const float *X, int T, const uint8_t *idx,
                   const uint16_t *scale, const float *books, int M, int N, int cb_base,
                   void *stream);

/* 0 when no tensor-core kernel of this library has given up a bounded wait
 * since the last clear; WARP_E_TIMEOUT otherwise.  clear = 1 resets the
 * flag.  Synchronous (reads a device flag). */
WARP_API int warp_umma_status(int clear);

/* Dequantized VQ3R matrix, fp32 [M][N]: recon = ((0 + C0[i0]) + C1[i1]) +
 * C2[i2] per dimension times f16(scale[r]) (tools/kimi_ref.py:262-270, books
 * decoded as src/model.c:2916-2922).  books is [n_books][256][8] fp32.
 * Bit-exact. */
WARP_API int warp_vq_dequant(float *W, const uint8_t *idx, const uint16_t *scale,
                    const float *books, int M, int N, int cb_base, void *stream);

/* RVQ encoder, waste_vq_encode (src/vq.c:50-105): X [n][8] fp32, books
 * [stages][256][8] fp32 -> codes [n][stages], nearest centroid by squared
 * L2 summed in d order, lowest index on ties.  Bit-exact. */
WARP_API int warp_vq_encode(const float *X, int64_t n, const float *books, int stages,
                   uint8_t *codes, void *stream);

/* Softmax top-k router, waste_qwen_moe_route (src/qwen_moe.c:10-44), for T
 * tokens: logits [T][E] -> idx [T][K], w [T][K] in selection order. */
WARP_API int warp_qwen_route(const float *logits, int T, int E, int K, int renorm,
                    int *idx, float *w, void *stream);

/* moe_layer's routing (src/model.c:5466-5556) for T tokens: logits [T][E]
 * -> idx [T][K], w [T][K] in selection order.  Scores by score_func (0
 * sigmoid, 1 softmax, 2 sqrt-softplus: router_scores, model.c:5466-5486);
 * K passes take the strictly greatest score + bias among unused experts
 * (lowest id on ties; bias NULL = 0, it moves the ranking only); w is the
 * unbiased score, divided by (sum of the K + 1e-20) with renorm, then times
 * routed_scale. */
WARP_API int warp_moe_route(const float *logits, int T, int E, int K, int score_func,
                   const float *bias, int renorm, float routed_scale, int *idx, float *w,
                   void *stream);

/* waste_rmsnorm (src/model.c:178-184) over `rows` rows of n: o = x *
 * 1/sqrtf(mean(x^2) + eps) * w (w NULL = 1).  In-place allowed. */
WARP_API int warp_rmsnorm(const float *x, const float *w, float *o, int rows, int n,
                          float eps, void *stream);

/* ---- resident MoE layer ---------------------------------------------------------- */

typedef struct warp_moe_layer warp_moe_layer;

/* Geometry and weights of one MoE layer, all DEVICE pointers.
 *   bank       E expert records of rec_bytes each, contiguous and sorted by
 *              expert id — the experts-L{n}.bin layout (FORMAT.md "Expert bank
 *              record"); record offsets are read from the headers.
 *   booksT     the layer's codebooks [n_books][8][256] fp32; books the same
 *              [n_books][256][8] (both decoded as src/model.c:2911-2941).
 *   router     fp32 [E][hidden] gate matrix.
 *   shared_*   the shared expert, Q4G/Q8G trunk tensors (NULL for none):
 *              gate/up [shared_inter][hidden], down [hidden][shared_inter].
 *   shared_gate fp32 [hidden] sigmoid gate (qwen_moe_layer), or NULL for an
 *              unscaled add (moe_layer). */
typedef struct {
    int hidden, inter, n_experts, top_k, renorm;
    const uint8_t *bank;
    size_t rec_bytes;
    const float *booksT, *books;
    int n_books;
    const float *router;
    const void *shared_gate_w, *shared_up_w, *shared_down_w;
    const uint16_t *shared_gate_s, *shared_up_s, *shared_down_s;
    int shared_inter, shared_group, shared_bits;
    const float *shared_gate;
    /* 1: re-tile the bank's index blocks in place, once, into the device tile
     * layout the decode gather reads with fully coalesced loads (headers get
     * flags bit 0x80; a bank already marked is used as is).  The bank then
     * no longer holds container-layout index blocks.  0: read the container
     * layout directly (slower). */
    int tile_bank;
    /* Expert parallelism over ep_size ranks (0 or 1: off).  Rank ep_rank owns
     * the experts e with e % ep_size == ep_rank; its bank holds just those,
     * in increasing e (record x is expert x*ep_size + ep_rank), while the
     * router, codebooks and shared expert are the whole layer's.  A layer
     * created with ep_size > 1 runs through warp_moe_layer_forward_ep and
     * warp_moe_layer_combine. */
    int ep_rank, ep_size;
    /* Tokens warp_moe_layer_prefill takes at most (0: no prefill workspace).
     * Prefill needs a Q4 shared expert (shared_bits 4) when one is given. */
    int prefill_tokens;
    /* The router.  router_kind 0: Qwen's softmax top-k
     * (waste_qwen_moe_route, src/qwen_moe.c:10-44; renorm as above).
     * router_kind 1: moe_layer's (src/model.c:5466-5556): scores by
     * score_func (0 sigmoid, 1 softmax, 2 sqrt-softplus, the numbering of
     * src/model.h:179-181), score_bias (fp32 [n_experts], added for the
     * selection only; NULL for none), weights renormalised by their sum +
     * 1e-20 when renorm is set, then multiplied by routed_scale. */
    int router_kind, score_func;
    const float *score_bias;
    float routed_scale;
    /* How an expert-parallel layer (ep_size > 1) splits the routed experts.
     * 0: by expert id, as described at ep_rank above.  1: every rank's bank
     * holds all n_experts records (replicated), and the routes of a step are
     * dealt in route order: rank r computes route t*top_k + j when
     * (t*top_k + j) % ep_size == r, which balances the ranks exactly. */
    int ep_mode;
} warp_moe_desc;

/* Validates the geometry and the records' headers (magic, fmt, offsets) and
 * allocates the layer's workspace for up to max_tokens tokens. */
WARP_API int warp_moe_layer_create(const warp_moe_desc *d, int max_tokens,
                          warp_moe_layer **out);
WARP_API void warp_moe_layer_destroy(warp_moe_layer *L);

/* Synchronizes `stream` and reports a device-side failure recorded by the
 * layer's kernels since creation (0 = none). */
WARP_API int warp_moe_layer_status(warp_moe_layer *L, void *stream);

/* One MoE layer for T tokens, device pointers: out[t] = sum_j w[t][j] *
 * expert_{idx[t][j]}(x[t]) (route order) + sg * shared(x[t]).  When
 * residual is non-NULL, out[t] also gets residual[t] added first.  idx/w
 * (optional, [T][K]) receive the routing.  A layer owns one workspace:
 * calls on the same layer (forward, forward_ep, combine, prefill) must not
 * overlap on the device, so issue them on one stream or order them with
 * events. */
WARP_API int warp_moe_layer_forward(warp_moe_layer *L, const float *x, int T,
                           const float *residual, float *out, int *idx,
                           float *w, void *stream);

/* The decoder block's MoE half for T tokens: out[t] = h[t] + MoE(x[t]) with
 * x[t] = waste_rmsnorm(h[t]) (src/model.c:178-184: r = 1 / sqrtf(sum h^2 /
 * n + eps), x = h * r * norm_w, norm_w NULL = 1) -- the residual stream of a
 * decoder layer whose attention half is the identity.  warp_rmsnorm into
 * the layer's own buffer, then warp_moe_layer_forward(x, residual = h), on
 * `stream`.  out must be another buffer than h; h and norm_w 16-byte
 * aligned. */
WARP_API int warp_moe_block_forward(warp_moe_layer *L, const float *h, int T,
                           const float *norm_w, float eps, float *out, int *idx,
                           float *w, void *stream);

/* Expert-parallel forward, first half (no host synchronisation).  For T
 * tokens x [T][hidden] (the same on every rank) it routes every token, runs
 * the routes this rank computes (ep_mode), and writes slots [T][S][hidden]
 * fp32, S = warp_moe_layer_slots_per_token:
 *   slot (t, j < top_k)  route j's unweighted output (chunk-summed down rows
 *                        times their row scales) when this rank computes it,
 *                        else 0;
 *   slot (t, top_k + b)  partial b of the shared expert: its down projection
 *                        over column block b of nb (S = top_k + nb; nb = 8
 *                        when shared_inter is a multiple of 8 groups), for
 *                        the blocks b in [nb*r/n, nb*(r+1)/n) this rank
 *                        computes (with the gate/up rows feeding them), else 0.
 * Every slot has exactly one non-zero contributor, so an all-reduce (sum) of
 * the slots over the ranks is exact in any order; warp_moe_layer_combine
 * then finishes the layer identically on every rank, and the result equals
 * warp_moe_layer_forward's on one GPU bit for bit (which sums the same
 * shared-expert partials in the same order).  The combine of
 * model.c:5858-5869 (route-ordered sum) is what this decomposition keeps. */
WARP_API int warp_moe_layer_forward_ep(warp_moe_layer *L, const float *x, int T,
                              float *slots, int *idx, float *w, void *stream);

/* The layer for T tokens at once (prefill, T <= prefill_tokens), on the
 * tensor cores: route every token (as forward does), group the routes by
 * expert, run each touched expert once over its tokens as tcgen05 GEMMs
 * (gate and up with the SwiGLU in the epilogue, then down; weights
 * dequantized to fp16 tiles in shared memory, fp32 accumulation), a Q4
 * shared expert the same way over all tokens (another format through the
 * trunk matmul, 64 tokens a launch), and combine in route order —
 * moe_chunk (src/model.c:7110-7290) reads each distinct expert once the
 * same way.  Outputs agree with the fp32 reference within 2e-3 relative L2;
 * routing is the exact top-k.  No host synchronisation.  Not for
 * expert-parallel layers. */
WARP_API int warp_moe_layer_prefill(warp_moe_layer *L, const float *x, int T,
                           const float *residual, float *out, int *idx, float *w,
                           void *stream);

/* Second half: out[t] = residual[t] + sum_j w[t][j] * slot(t, j) (route
 * order) + sg[t] * (sum_b slot(t, top_k + b), in b order), with the routing
 * of the last warp_moe_layer_forward_ep on this layer.  residual may be
 * NULL. */
WARP_API int warp_moe_layer_combine(warp_moe_layer *L, const float *slots, int T,
                           const float *residual, float *out, void *stream);

/* S, the slots per token of forward_ep / combine: top_k plus the shared
 * expert's column blocks (0 without a shared expert). */
WARP_API int warp_moe_layer_slots_per_token(warp_moe_layer *L);

/* Phase timing for measurement runs: with on = 1 every eager forward records
 * CUDA events around its phases on the caller's stream and waits for the last
 * one; warp_moe_layer_timings writes the accumulated
 * milliseconds of router, gate/up gather, SwiGLU, down gather, shared expert
 * and combine into ms[6] and returns how many forwards they cover. */
WARP_API int warp_moe_layer_set_timing(warp_moe_layer *L, int on);
WARP_API int warp_moe_layer_timings(warp_moe_layer *L, double *ms);
/* With timing on, a forward captured into a CUDA graph records its phase
 * events as external event nodes; after each replay, collect adds that
 * replay's phase times to the totals. */
WARP_API int warp_moe_layer_collect(warp_moe_layer *L);

#ifdef __cplusplus
}
#endif
#endif /* WARP_CUDA_H */
