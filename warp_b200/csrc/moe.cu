// moe.cu — one resident MoE layer: router, routed VQ3R experts, shared
// expert, route-ordered combine.  Everything runs on the caller's stream
// with no host synchronization, so a whole decode step can be captured in a
// CUDA graph.
//
// Per token the data flow is the reference's (qwen_moe_layer,
// model.c:8180-8405; moe_layer, model.c:5488-5940):
//   router -> top-k -> gate/up tables from x (shared by all K experts) ->
//   gate/up gather -> SwiGLU -> down table per expert -> down gather ->
//   out = sum_j w_j * acc_j in route order + sg * shared expert.
#include "common.cuh"
#include "moe_prefill.cuh"
#include "mvq.cuh"
#include "router.cuh"
#include "vq_gather.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

namespace warp {

// The 48-byte WEXP header (waste_format.h:98-130).
struct ExpertHdr {
    uint32_t magic;
    uint16_t layer, expert_id;
    uint8_t fmt, flags;
    uint16_t codebook_id, lowrank_id, reserved0;
    uint32_t rec_4k_blocks, gate_off, up_off, down_off, chan_corr_off, crc32;
    uint32_t reserved1[2];
};
static_assert(sizeof(ExpertHdr) == 48, "expert header layout");

// Header flags bit of a record whose index blocks were re-tiled in device
// memory (bank_tile).  The container's own flags use bits 0-2
// (waste_format.h:84-86); a device bank is never written back to disk.
constexpr uint8_t kFlagTiled = 0x80;

__global__ void mark_tiled_kernel(uint8_t *bank, size_t rec_bytes, int E) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e < E) bank[(size_t)e * rec_bytes + 9] |= kFlagTiled;   // flags byte
}

// SwiGLU and the down tables, two CTAs per (route r, chunk c of the down
// input).  Each computes h = silu(g) * u for the chunk's 256 inputs, with
// g, u the chunk-summed gate/up rows times their fp16 row scales (vq_rows'
// final multiply, model.c:3974-3976; SwiGLU model.c:1231, 1264) — four
// threads per input, each summing every fourth chunk partial — and then
// half of the table of those 32 positions (the down codebooks, cb0 + 6)
// as part of a compact image: the down LUT build of vq_matvec
// (model.c:4140-4149), once per route.
constexpr int kMidThreads = 1024;
constexpr int kMidSplit = 2;

__global__ void __launch_bounds__(kMidThreads)
moe_mid_kernel(const float *__restrict__ pgu, int nch_gu, size_t chunk_stride,
               const int *__restrict__ idx, const uint8_t *__restrict__ bank,
               size_t rec_bytes, uint32_t sc_off, int K, int inter,
               const float *__restrict__ books, int cb_down, int nch_d,
               uint32_t *__restrict__ images, const int *__restrict__ plan,
               int max_routes) {
    __shared__ __align__(16) float sb[kSt * kEnt * kVec];
    __shared__ float hx[kChunk * kVec];
    const int seg = blockIdx.x / kMidSplit, part = blockIdx.x % kMidSplit;
    const int r = seg / nch_d, c = seg % nch_d;
    // route r of the step, or work route r of this rank (plan): the gate/up
    // partials of a work route sit at groups 2r, 2r + 1 (one matrix each)
    int route = r, rec;
    if (plan) {
        if (r >= plan[0]) return;                       // block-uniform
        route = plan[1 + r];
        rec = plan[1 + max_routes + r];
    } else {
        rec = idx[r];
    }
    const int t = route / K, j = route % K;
    const float4 *src = (const float4 *)(books + (size_t)cb_down * kEnt * kVec);
    for (int i = threadIdx.x; i < kSt * kEnt * kVec / 4; i += kMidThreads)
        ((float4 *)sb)[i] = src[i];
    const int q = threadIdx.x >> 2, lane4 = threadIdx.x & 3;
    const int i = c * kChunk * kVec + q;                // input index of the down matrix
    const bool ok = i < inter;
    // the books, the routing and the row scales are older than the gate/up
    // gather before this kernel: they are read before the wait, its
    // partials after it
    float sg_ = 0.0f, su_ = 0.0f;
    if (ok && lane4 == 0) {
        const uint16_t *sc = (const uint16_t *)(bank + (size_t)rec * rec_bytes + sc_off);
        sg_ = f16_to_f32(sc[i]);
        su_ = f16_to_f32(sc[inter + i]);
    }
    pdl_wait();
    pdl_trigger();
    float g = 0.0f, u = 0.0f;
    if (ok) {
        const size_t og = plan ? (size_t)(2 * r) * inter + i
                               : ((size_t)(t * 2 + 0) * K + j) * inter + i;
        const size_t ou = og + (plan ? (size_t)inter : (size_t)K * inter);
#pragma unroll 4
        for (int cc = lane4; cc < nch_gu; cc += 4) {
            g += pgu[cc * chunk_stride + og];
            u += pgu[cc * chunk_stride + ou];
        }
    }
    g += __shfl_xor_sync(0xffffffffu, g, 1);
    u += __shfl_xor_sync(0xffffffffu, u, 1);
    g += __shfl_xor_sync(0xffffffffu, g, 2);
    u += __shfl_xor_sync(0xffffffffu, u, 2);
    if (lane4 == 0) {
        float h = 0.0f;
        if (ok) {
            g *= sg_;
            u *= su_;
            h = (g / (1.0f + expf(-g))) * u;
        }
        hx[q] = h;
    }
    __syncthreads();
    const int p = threadIdx.x & 31;
    float xv[kVec];
#pragma unroll
    for (int d = 0; d < kVec; d++) xv[d] = hx[p * kVec + d];
    uint32_t *img = images + (size_t)seg * kImageWords;
    const int w0 = part * (kImageWords / kMidSplit), w1 = w0 + kImageWords / kMidSplit;
#pragma unroll 2
    for (int w = w0 + threadIdx.x; w < w1; w += kMidThreads) {
        int s, code;
        if (w < 16384) { code = w >> 6; s = (w >> 5) & 1; }
        else { code = (w - 16384) >> 5; s = 2; }
        img[w] = __float_as_uint(lut_entry(xv, sb + (s * kEnt + code) * kVec));
    }
}

// out[t][i] = (residual) + sum_j w[t][j] * y_j[i] (route order, multiply then
// add, model.c:8385-8400) + sg[t] * shared[t][i] (model.c:8402-8404).
// A CTA owns 32 columns of one token: first every (route, column) pair sums
// its chunk partials and applies the row scale in parallel, then one thread
// per column adds the routes in order.
constexpr int kCombineCols = 32;

__global__ void moe_combine_kernel(const float *__restrict__ pd, int nch,
                                   size_t chunk_stride,
                                   const int *__restrict__ idx,
                                   const float *__restrict__ w,
                                   const uint8_t *__restrict__ bank,
                                   size_t rec_bytes, uint32_t sc_off, int T,
                                   int K, int inter, int hid,
                                   const float *__restrict__ shared, int nsh,
                                   size_t sh_stride, const float *__restrict__ sg,
                                   const float *__restrict__ residual,
                                   float *__restrict__ out) {
    __shared__ float ys[64][kCombineCols];
    const int tiles = (hid + kCombineCols - 1) / kCombineCols;
    const int t = blockIdx.x / tiles;
    const int i0 = (blockIdx.x % tiles) * kCombineCols;
    const int lane = threadIdx.x & 31;
    const int i = i0 + lane;
    const size_t q = (size_t)t * hid + i;
    // everything but the down partials is older than the down gather before
    // this kernel (routing, weights, row scales, the shared expert joined
    // before the launch, the residual): read before the wait
    const int j0 = threadIdx.x >> 5;
    float sc0 = 0.0f;
    if (j0 < K && i < hid) {
        const uint16_t *sc = (const uint16_t *)(bank + (size_t)idx[t * K + j0] * rec_bytes + sc_off);
        sc0 = f16_to_f32(sc[2 * inter + i]);
    }
    // the shared expert: its column-block partials added in block order
    float sh = 0.0f, res = 0.0f, sgt = 0.0f;
    if (threadIdx.x < 32 && i < hid) {
        if (shared) {
            for (int b = 0; b < nsh; b++) sh = __fadd_rn(sh, shared[(size_t)b * sh_stride + q]);
            sgt = sg[t];
        }
        if (residual) res = residual[q];
    }
    pdl_wait();                                   // the down partials
    pdl_trigger();
    for (int j = j0; j < K; j += blockDim.x >> 5) {
        float y = 0.0f;
        if (i < hid) {
            const int r = t * K + j;
            float s = sc0;
            if (j != j0) {
                const uint16_t *sc = (const uint16_t *)(bank + (size_t)idx[r] * rec_bytes + sc_off);
                s = f16_to_f32(sc[2 * inter + i]);
            }
#pragma unroll 8
            for (int c = 0; c < nch; c++) y += pd[c * chunk_stride + (size_t)r * hid + i];
            y *= s;
        }
        ys[j][lane] = y;
    }
    __syncthreads();
    if (threadIdx.x >= 32 || i >= hid) return;
    float acc = 0.0f;
    for (int j = 0; j < K; j++) acc = __fadd_rn(acc, __fmul_rn(w[t * K + j], ys[j][lane]));
    if (shared) acc = __fadd_rn(acc, __fmul_rn(sgt, sh));
    out[q] = residual ? __fadd_rn(res, acc) : acc;
}

// Expert parallelism: this rank's work routes, in route order.  One CTA
// scans the T*K routes in blocks of kPlanThreads with a ballot + warp scan:
// plan[0] = count, plan[1 + p] = route, plan[1 + max_routes + p] = record
// index in the local bank (expert / ep_size when the bank holds this rank's
// experts; the expert id when routes are dealt over a replicated bank),
// inv[route] = p or -1.
constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads)
ep_plan_kernel(const int *__restrict__ idx, int n, int rank, int size, int deal,
               int *__restrict__ plan, int max_routes, int *__restrict__ inv) {
    __shared__ int wsum[kPlanThreads / 32];
    __shared__ int base_s;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (threadIdx.x == 0) base_s = 0;
    __syncthreads();
    for (int b0 = 0; b0 < n; b0 += kPlanThreads) {
        const int r = b0 + threadIdx.x;
        const int e = r < n ? idx[r] : -1;
        // deal: routes dealt in route order over a replicated bank; else
        // the experts this rank holds
        const bool own = e >= 0 && (deal ? r % size == rank : e % size == rank);
        const unsigned bal = __ballot_sync(0xffffffffu, own);
        if (lane == 0) wsum[w] = __popc(bal);
        __syncthreads();
        if (w == 0) {
            int v = wsum[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += u;
            }
            wsum[lane] = v;                             // inclusive
        }
        __syncthreads();
        const int pos = base_s + (w ? wsum[w - 1] : 0) + __popc(bal & ((1u << lane) - 1u));
        if (own) {
            plan[1 + pos] = r;
            plan[1 + max_routes + pos] = deal ? e : e / size;
        }
        if (r < n) inv[r] = own ? pos : -1;
        const int tot = wsum[kPlanThreads / 32 - 1];
        __syncthreads();
        if (threadIdx.x == 0) base_s += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) plan[0] = base_s;
}

// slots[t][j][i] for j < K: the chunk-summed down partials of route (t, j)
// times the row scale — exactly moe_combine_kernel's per-route value — when
// this rank computes the route, else 0.  slots[t][K + b][i], the shared
// expert's column-block partials, = 0 for the blocks another rank computes
// (outside [b0, b1)); this rank's are written by the block matvec.
__global__ void moe_slots_kernel(const float *__restrict__ pd, int nch, size_t chunk_stride,
                                 const int *__restrict__ plan, int max_routes,
                                 const int *__restrict__ inv,
                                 const uint8_t *__restrict__ bank, size_t rec_bytes,
                                 uint32_t sc_off, int T, int K, int nsh, int inter, int hid,
                                 int b0, int b1, float *__restrict__ slots) {
    const size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int S = K + nsh;
    if (q >= (size_t)T * S * hid) return;
    const int i = (int)(q % hid);
    const int tj = (int)(q / hid);
    const int t = tj / S, j = tj % S;
    if (j >= K) {
        const int b = j - K;
        if (b < b0 || b >= b1) slots[q] = 0.0f;
        return;
    }
    const int r = inv[t * K + j];
    float y = 0.0f;
    if (r >= 0) {
        const uint16_t *sc = (const uint16_t *)(bank + (size_t)plan[1 + max_routes + r] *
                                                           rec_bytes + sc_off);
#pragma unroll 8
        for (int c = 0; c < nch; c++) y += pd[c * chunk_stride + (size_t)r * hid + i];
        y *= f16_to_f32(sc[2 * inter + i]);
    }
    slots[q] = y;
}

// out[t][i] from the all-reduced slots, in moe_combine_kernel's order:
// route-ordered multiply-then-add, then the gated shared expert, then the
// residual.
// (S slots per token: K routes, then nsh <= S - K shared-expert partials
// added in order; nsh = 0 for a layer without one)
__global__ void moe_combine_slots_kernel(const float *__restrict__ slots,
                                         const float *__restrict__ w, int T, int K, int S,
                                         int hid, int nsh, const float *__restrict__ sg,
                                         const float *__restrict__ residual,
                                         float *__restrict__ out) {
    const size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= (size_t)T * hid) return;
    const int t = (int)(q / hid), i = (int)(q % hid);
    const float *s = slots + (size_t)t * S * hid + i;
    float acc = 0.0f;
    for (int j = 0; j < K; j++) acc = __fadd_rn(acc, __fmul_rn(w[t * K + j], s[(size_t)j * hid]));
    if (nsh > 0) {
        float sh = 0.0f;
        for (int b = 0; b < nsh; b++) sh = __fadd_rn(sh, s[(size_t)(K + b) * hid]);
        acc = __fadd_rn(acc, __fmul_rn(sg[t], sh));
    }
    out[q] = residual ? __fadd_rn(residual[q], acc) : acc;
}

}  // namespace warp

using namespace warp;

struct warp_moe_layer {
    warp_moe_desc d;
    int max_tokens;
    int cb0;
    bool tiled;             // index blocks in the device tile layout
    uint32_t off[4];        // gate, up, down, scales
    int nch_gu, nch_d;
    // workspace (one allocation)
    void *ws;
    float *rpart, *rparts, *w, *sg, *pgu, *pd, *sh_y, *sh_out, *xn;
    unsigned *ticket;           // router_kernel's last-CTA counter (0 between launches)
    unsigned *pf_ticket;        // the same for the prefill router, so the two never share one
    float *pf_sq_y;             // prefill, non-Q4 shared expert: [64][2 si] gate | up
    void *pf_sq_xf;             //   and the trunk matmul's scratch
    uint32_t *img_gu, *img_d;   // table images: gate/up per (token, kind, chunk), down per (route, chunk)
    int *idx, *err;
    int *plan, *inv;            // expert-parallel work routes (ep_plan_kernel)
    int ep_rank, ep_size, E_loc, ep_mode;
    int nsh;                    // the shared expert's column blocks (0: no shared expert)
    float *sh_part;             // [T][hidden] its output, the blocks folded (one GPU)
    // phase timing (eager runs only): events at the phase boundaries and the
    // accumulated milliseconds per phase
    bool timing;
    cudaEvent_t ev[8];
    double phase_ms[8];
    int phase_n;
    // The table images and the shared expert depend on x only: they run, in
    // that order, on a side stream forked from the caller's stream at the
    // start of a forward; the gate/up gather waits for the images and the
    // combine for the shared expert (under stream capture the fork and the
    // joins become a parallel branch of the graph).  One side stream rather
    // than two: the images then never queue behind the shared expert's CTAs,
    // which measured faster than running the two concurrently.
    cudaStream_t side;
    cudaEvent_t ev_fork, ev_img, ev_shared;
    // prefill workspace (prefill_tokens > 0), one allocation
    int pf_tokens, pf_items;
    void *pf_ws;
    float *pf_slots, *pf_logits, *pf_parts, *pf_w, *pf_sg;
    uint16_t *pf_h, *pf_hs, *pf_xh;
    int *pf_idx, *pf_counts, *pf_offsets, *pf_slot_route, *pf_items_buf;
};

// The layer's router, as its descriptor names it.
static RouteCfg route_cfg(const warp_moe_desc &d) {
    RouteCfg rc;
    rc.kind = d.router_kind == 1 ? 1 : 0;
    rc.func = d.score_func;
    rc.bias = d.score_bias;
    rc.scale = d.routed_scale;
    return rc;
}

// Phases of one forward, in launch order.
enum { PH_ROUTER, PH_GATEUP, PH_MID, PH_DOWN, PH_SHARED, PH_COMBINE, PH_N };

// Record phase boundary i.  Under stream capture the record becomes an
// external event node of the graph, so every replay times the phases on the
// device; warp_moe_layer_collect reads them after the replay finished.
static void mark(warp_moe_layer *L, int i, cudaStream_t st) {
    if (!L->timing) return;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs == cudaStreamCaptureStatusActive)
        cudaEventRecordWithFlags(L->ev[i], st, cudaEventRecordExternal);
    else
        cudaEventRecord(L->ev[i], st);
}

static void collect(warp_moe_layer *L) {
    cudaEventSynchronize(L->ev[PH_N]);
    for (int i = 0; i < PH_N; i++) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, L->ev[i], L->ev[i + 1]);
        L->phase_ms[i] += ms;
    }
    L->phase_n++;
}

extern "C" int warp_moe_layer_create(const warp_moe_desc *d, int max_tokens,
                                     warp_moe_layer **out) {
    WARP_ARG(d && out && max_tokens >= 1, "moe_layer_create: bad arguments");
    *out = nullptr;
    const int hid = d->hidden, inter = d->inter, E = d->n_experts, K = d->top_k;
    WARP_ARG(hid > 0 && hid % 8 == 0 && inter > 0 && inter % 8 == 0,
             "moe: hidden and inter must be multiples of 8");
    WARP_ARG(E >= 1 && E <= 384 && K >= 1 && K <= E && K <= 64,
             "moe: need 1 <= top_k <= n_experts <= 384");
    WARP_ARG(d->router_kind == 0 || (d->router_kind == 1 && d->score_func >= 0 &&
                                     d->score_func <= 2),
             "moe: router_kind must be 0 or 1, score_func 0..2");
    WARP_ARG(d->bank && d->booksT && d->books && d->router && d->rec_bytes >= 48,
             "moe: missing bank, codebooks or router");
    WARP_ARG(((uintptr_t)d->bank & 15) == 0 && d->rec_bytes % 16 == 0,
             "moe: bank must be 16-byte aligned with a record size multiple of 16");
    WARP_ARG(((uintptr_t)d->books & 15) == 0, "moe: books must be 16-byte aligned");
    if (d->shared_gate_w)
        WARP_ARG(d->shared_up_w && d->shared_down_w && d->shared_gate_s &&
                     d->shared_up_s && d->shared_down_s && d->shared_inter > 0,
                 "moe: incomplete shared expert");
    const int ep_size = d->ep_size > 1 ? d->ep_size : 1;
    const int ep_rank = ep_size > 1 ? d->ep_rank : 0;
    WARP_ARG(ep_rank >= 0 && ep_rank < ep_size && ep_size <= E,
             "moe: need 0 <= ep_rank < ep_size <= n_experts");
    WARP_ARG(d->ep_mode == 0 || d->ep_mode == 1, "moe: ep_mode must be 0 or 1");
    const int ep_mode = ep_size > 1 ? d->ep_mode : 0;
    // records this rank holds: experts ep_rank, ep_rank + ep_size, ... (mode
    // 0), or all of them (mode 1: routes dealt over a replicated bank)
    const int E_loc = ep_mode == 1 ? E : (E - ep_rank + ep_size - 1) / ep_size;
    int rc = gather_setup();
    if (rc) return rc;

    // Headers: every record must be a VQ3R expert of this geometry with the
    // same offsets and codebook base (what record_check, model.c:3645,
    // requires of a bank).
    std::vector<ExpertHdr> hdr(E_loc);
    cudaError_t e = cudaMemcpy2D(hdr.data(), sizeof(ExpertHdr), d->bank, d->rec_bytes,
                                 sizeof(ExpertHdr), E_loc, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "moe: reading record headers");
    const size_t idx_gu = (size_t)((inter + 63) / 64) * (hid / 8) * 64 * 3;
    const size_t idx_d = (size_t)((hid + 63) / 64) * (inter / 8) * 64 * 3;
    const bool was_tiled = (hdr[0].flags & kFlagTiled) != 0;
    for (int x = 0; x < E_loc; x++) {
        const ExpertHdr &h = hdr[x];
        const int want_id = ep_mode == 1 ? x : x * ep_size + ep_rank;
        if (h.magic != 0x50584557u || h.fmt != 4 || h.expert_id != want_id ||
            ((h.flags & kFlagTiled) != 0) != was_tiled ||
            h.codebook_id != hdr[0].codebook_id || h.gate_off != hdr[0].gate_off ||
            h.up_off != hdr[0].up_off || h.down_off != hdr[0].down_off ||
            h.chan_corr_off != hdr[0].chan_corr_off) {
            set_error("moe: record %d is not a VQ3R expert matching record 0", x);
            return WARP_E_FORMAT;
        }
    }
    const ExpertHdr &h0 = hdr[0];
    if (h0.gate_off % 16 || h0.up_off % 16 || h0.down_off % 16 || h0.chan_corr_off % 2 ||
        h0.up_off < h0.gate_off + idx_gu || h0.down_off < h0.up_off + idx_gu ||
        h0.chan_corr_off < h0.down_off + idx_d ||
        h0.chan_corr_off + (size_t)2 * (2 * inter + hid) > d->rec_bytes ||
        (size_t)h0.codebook_id + 9 > (size_t)d->n_books) {
        set_error("moe: record offsets do not fit hidden %d / inter %d", hid, inter);
        return WARP_E_FORMAT;
    }

    warp_moe_layer *L = new (std::nothrow) warp_moe_layer();
    if (!L) return WARP_E_NOMEM;
    L->d = *d;
    L->max_tokens = max_tokens;
    L->cb0 = h0.codebook_id;
    L->off[0] = h0.gate_off;
    L->off[1] = h0.up_off;
    L->off[2] = h0.down_off;
    L->off[3] = h0.chan_corr_off;
    L->tiled = was_tiled || d->tile_bank;
    L->ep_rank = ep_rank;
    L->ep_size = ep_size;
    L->E_loc = E_loc;
    L->ep_mode = ep_mode;
    // The shared expert's down projection runs in nsh fixed column blocks
    // (8 when its width allows, each a whole number of groups), summed in
    // block order by the combine: the unit an expert-parallel rank takes.
    L->nsh = 0;
    if (d->shared_gate_w) {
        L->nsh = 1;
        for (int nb = 8; nb >= 1; nb >>= 1)
            if (d->shared_inter % (nb * d->shared_group) == 0) { L->nsh = nb; break; }
    }
    if (d->tile_bank && !was_tiled) {
        // re-tile gate, up and down of every record, then mark the headers
        uint8_t *bank = (uint8_t *)d->bank;
        // A failure after the first kind was re-tiled leaves a bank that is
        // neither layout and carries no mark: say so, the caller must reload it.
        if ((rc = bank_tile(bank, d->rec_bytes, h0.gate_off, inter, hid / 8, E_loc, 0)) ||
            (rc = bank_tile(bank, d->rec_bytes, h0.up_off, inter, hid / 8, E_loc, 0)) ||
            (rc = bank_tile(bank, d->rec_bytes, h0.down_off, hid, inter / 8, E_loc, 0))) {
            delete L;
            char why[512];
            snprintf(why, sizeof why, "%s", warp_last_error());
            set_error("moe: re-tiling the bank failed part way (%s); the bank may be "
                      "partly re-tiled and must be reloaded before another create", why);
            return rc;
        }
        mark_tiled_kernel<<<cdiv(E_loc, 256), 256>>>(bank, d->rec_bytes, E_loc);
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            delete L;
            set_error("moe: re-tiling the bank failed (%s); the bank may be partly "
                      "re-tiled and must be reloaded before another create",
                      cudaGetErrorString(e));
            return WARP_E_CUDA;
        }
    }
    L->nch_gu = (hid / 8 + kChunk - 1) / kChunk;
    L->nch_d = (inter / 8 + kChunk - 1) / kChunk;
    const int T = max_tokens;
    const int si = d->shared_gate_w ? d->shared_inter : 0;
    const size_t n_rpart = (size_t)T * (E + 1);
    const size_t n_img_gu = (size_t)T * 2 * L->nch_gu * kImageWords;
    const size_t n_img_d = (size_t)T * K * L->nch_d * kImageWords;
    const size_t n_w = (size_t)T * K;
    const size_t n_sg = T;
    const size_t n_pgu = (size_t)L->nch_gu * T * 2 * K * inter;
    const size_t n_pd = (size_t)L->nch_d * T * K * hid;
    const size_t n_shy = (size_t)T * 2 * si;
    const size_t n_sho = (size_t)T * hid;
    const size_t n_shp = (size_t)(si ? 1 : 0) * T * hid;
    const size_t floats = 3 * n_rpart + n_sho + n_img_gu + n_img_d + n_w + n_sg + n_pgu + n_pd +
                          n_shy + n_sho + n_shp;
    const size_t bytes = floats * 4 + n_w * 4 + 64 + 16 * 16 + (1 + 3 * n_w) * 4 + 64;
    e = cudaMalloc(&L->ws, bytes);
    if (e != cudaSuccess) { delete L; return cuda_fail(e, "moe workspace"); }
    float *p = (float *)L->ws;
    auto take = [&](size_t n) { float *r = p; p += (n + 3) & ~(size_t)3; return r; };
    L->rpart = take(n_rpart);
    L->rparts = take(2 * n_rpart);
    L->xn = take(n_sho);
    L->img_gu = (uint32_t *)take(n_img_gu);
    L->img_d = (uint32_t *)take(n_img_d);
    L->w = take(n_w);
    L->sg = take(n_sg);
    L->pgu = take(n_pgu);
    L->pd = take(n_pd);
    L->sh_y = take(n_shy);
    L->sh_out = take(n_sho);
    L->sh_part = take(n_shp);
    L->idx = (int *)take(n_w);
    L->err = (int *)take(16);
    L->ticket = (unsigned *)(L->err + 8);
    L->pf_ticket = (unsigned *)(L->err + 9);
    L->plan = (int *)take(1 + 2 * n_w);
    L->inv = (int *)take(n_w);
    // The error word and the router's last-CTA tickets must read 0 before the
    // first kernel of any stream touches them: zero them and wait here, so a
    // caller on a non-blocking stream cannot run ahead of the clear.
    e = cudaMemset(L->err, 0, 16 * sizeof(int));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(L->ws);
        delete L;
        return cuda_fail(e, "moe: clearing the layer's status words");
    }
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&L->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->ev_fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->ev_img, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&L->ev_shared, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        warp_moe_layer_destroy(L);
        return cuda_fail(e, "moe: side streams");
    }
    if (d->prefill_tokens > 0) {
        const int Tp = d->prefill_tokens, R = Tp * K, si = d->shared_gate_w ? d->shared_inter : 0;
        if (ep_size > 1 || Tp > 128 * 65535) {
            warp_moe_layer_destroy(L);
            set_error("moe: prefill needs a single-GPU layer");
            return WARP_E_ARG;
        }
        // a shared expert other than Q4 runs through the trunk matmul, 64
        // tokens a launch: its [gate; up] outputs and the matmul's scratch
        const bool q8 = d->shared_gate_w && d->shared_bits != 4;
        const int sq_in = hid > si ? hid : si, sq_rows = 2 * si > hid ? 2 * si : hid;
        const size_t bytes_sq = q8 ? (size_t)kMvqMaxBatch * 2 * si * 4 +
                                         mvq_xf_bytes(kMvqMaxBatch, sq_in, sq_rows) + 512
                                   : 0;
        L->pf_tokens = Tp;
        L->pf_items = prefill_max_items(R, E);
        const size_t f_slots = (size_t)Tp * (K + 1) * hid, f_logits = (size_t)Tp * (E + 1);
        const size_t bytes_f = (f_slots + 3 * f_logits + (size_t)R + Tp) * 4;
        const size_t bytes_h = ((size_t)R * inter + (size_t)Tp * si + (size_t)Tp * hid) * 2;
        const size_t bytes_i = ((size_t)R + E + E + 1 + R + 1 + 3 * (size_t)L->pf_items) * 4;
        e = cudaMalloc(&L->pf_ws, bytes_f + bytes_h + bytes_i + bytes_sq + 16 * 256);
        if (e != cudaSuccess) {
            warp_moe_layer_destroy(L);
            return cuda_fail(e, "moe: prefill workspace");
        }
        uint8_t *q = (uint8_t *)L->pf_ws;
        auto grab = [&](size_t nbytes) { uint8_t *r = q; q += (nbytes + 255) & ~(size_t)255; return r; };
        L->pf_slots = (float *)grab(f_slots * 4);
        L->pf_logits = (float *)grab(f_logits * 4);
        L->pf_parts = (float *)grab(2 * f_logits * 4);
        L->pf_w = (float *)grab((size_t)R * 4);
        L->pf_sg = (float *)grab((size_t)Tp * 4);
        L->pf_h = (uint16_t *)grab((size_t)R * inter * 2);
        L->pf_hs = (uint16_t *)grab((size_t)Tp * si * 2 + 16);
        L->pf_xh = (uint16_t *)grab((size_t)Tp * hid * 2);
        L->pf_idx = (int *)grab((size_t)R * 4);
        L->pf_counts = (int *)grab((size_t)E * 4);
        L->pf_offsets = (int *)grab((size_t)(E + 1) * 4);
        L->pf_slot_route = (int *)grab((size_t)R * 4);
        L->pf_items_buf = (int *)grab((1 + 3 * (size_t)L->pf_items) * 4);
        if (q8) {
            L->pf_sq_y = (float *)grab((size_t)kMvqMaxBatch * 2 * si * 4);
            L->pf_sq_xf = grab(mvq_xf_bytes(kMvqMaxBatch, sq_in, sq_rows));
        }
    }
    *out = L;
    return WARP_OK;
}

extern "C" void warp_moe_layer_destroy(warp_moe_layer *L) {
    if (!L) return;
    if (L->timing)
        for (int i = 0; i < 8; i++) cudaEventDestroy(L->ev[i]);
    if (L->side) cudaStreamDestroy(L->side);
    if (L->pf_ws) cudaFree(L->pf_ws);
    if (L->ev_fork) cudaEventDestroy(L->ev_fork);
    if (L->ev_img) cudaEventDestroy(L->ev_img);
    if (L->ev_shared) cudaEventDestroy(L->ev_shared);
    cudaFree(L->ws);
    delete L;
}

// Fork the side stream off st: it waits for everything st has queued.
static int fork_side(warp_moe_layer *L, cudaStream_t st) {
    cudaError_t e = cudaEventRecord(L->ev_fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(L->side, L->ev_fork, 0);
    return e == cudaSuccess ? WARP_OK : cuda_fail(e, "moe: forking the side stream");
}

// Mark the side stream's work so far with `ev`.
static int mark_side(warp_moe_layer *L, cudaEvent_t ev) {
    cudaError_t e = cudaEventRecord(ev, L->side);
    return e == cudaSuccess ? WARP_OK : cuda_fail(e, "moe: side stream event");
}

// Make st wait for the side stream's work up to `ev`.
static int join_side(cudaEvent_t ev, cudaStream_t st) {
    cudaError_t e = cudaStreamWaitEvent(st, ev, 0);
    return e == cudaSuccess ? WARP_OK : cuda_fail(e, "moe: joining the side stream");
}

// The shared expert, in two steps over the same tokens x [T][hidden]:
//  * gate and up rows [r0, r1) in one matvec (a warp per row pair) into
//    sh_y [T][shared_inter] = silu(gate) * up, on the CUDA-core matvec,
//    whose per-row arithmetic does not depend on the rows or tokens a launch
//    carries;
//  * the down projection's column blocks [b0, b1) of nsh over sh_y into P
//    (mvq_blocks_launch): partial b of token t at P + b * pb +
//    t * pt, which the combine adds in block order; or, folded (all nsh
//    blocks on this GPU), their sum in that order at P + t * pt.
// An expert-parallel rank computes the blocks it owns (and the gate/up rows
// that feed them); one GPU computes all of them, to the same bits.
static int shared_gateup(warp_moe_layer *L, const float *x, int T, int r0, int r1,
                         cudaStream_t st) {
    const warp_moe_desc &d = L->d;
    const int hid = d.hidden, si = d.shared_inter;
    if (r1 <= r0) return WARP_OK;
    const int ng_h = (hid + d.shared_group - 1) / d.shared_group;
    const size_t rb = (size_t)ng_h * d.shared_group * d.shared_bits / 8;
    MvqArgs m = {};
    m.seg[0] = {(const uint8_t *)d.shared_gate_w + (size_t)r0 * rb,
                d.shared_gate_s + (size_t)r0 * ng_h, r1 - r0, 0};
    m.seg[1] = {(const uint8_t *)d.shared_up_w + (size_t)r0 * rb,
                d.shared_up_s + (size_t)r0 * ng_h, r1 - r0, 0};
    m.nseg = 2;
    m.pair = 1;                                 // a warp takes gate row r and up row r
    m.in = hid;
    m.group = d.shared_group;
    m.bits = d.shared_bits;
    m.rowbytes = rb;
    m.batch = T;
    m.X = x;
    m.Y = L->sh_y + r0;
    m.y_stride = si;
    return mvq_launch(m, st);
}

static int shared_down(warp_moe_layer *L, int T, int b0, int b1, bool fold, float *P,
                       long long pb, long long pt, cudaStream_t st) {
    const warp_moe_desc &d = L->d;
    const int si = d.shared_inter;
    const int ng_i = (si + d.shared_group - 1) / d.shared_group;
    MvqBlocks n = {};
    n.W = (const uint8_t *)d.shared_down_w;
    n.ws = d.shared_down_s;
    n.rows = d.hidden;
    n.in = si;
    n.group = d.shared_group;
    n.bits = d.shared_bits;
    n.rowbytes = (size_t)ng_i * d.shared_group * d.shared_bits / 8;
    n.nb = L->nsh;
    n.b0 = b0;
    n.b1 = b1;
    n.act_a = L->sh_y;                          // silu(gate) * up, [T][si]
    n.act_b = nullptr;
    n.act_stride = si;
    n.P = P;
    n.pb_stride = pb;
    n.pt_stride = pt;
    n.fold = fold;
    for (int t0 = 0; t0 < T; t0 += 16) {            // the block matvec takes 16 tokens a launch
        n.batch = T - t0 < 16 ? T - t0 : 16;
        n.act_a = L->sh_y + (size_t)t0 * si;
        n.P = P + (size_t)t0 * pt;
        const int rc = mvq_blocks_launch(n, st);
        if (rc) return rc;
    }
    return WARP_OK;
}

// One decode forward of T tokens.
static int forward_impl(warp_moe_layer *L, const float *x, int T, const float *residual,
                        float *out, int *idx_out, float *w_out, void *stream) {
    WARP_ARG(L && x && out && T >= 1 && T <= L->max_tokens,
             "moe_layer_forward: bad arguments");
    WARP_ARG(L->ep_size == 1,
             "moe_layer_forward: an expert-parallel layer runs through forward_ep + combine");
    WARP_ARG(((uintptr_t)x & 15) == 0, "moe_layer_forward: x must be 16-byte aligned");
    const warp_moe_desc &d = L->d;
    cudaStream_t st = (cudaStream_t)stream;
    const int hid = d.hidden, inter = d.inter, E = d.n_experts, K = d.top_k;
    int rc;
    mark(L, 0, st);
    const bool shared = d.shared_gate_w != nullptr;

    // 0. side stream: the gate/up tables of every token, then the shared
    // expert ([gate; up] in one matvec, then down over SwiGLU) — both depend
    // on x only
    if ((rc = fork_side(L, st))) return rc;
    if ((rc = lut_images(L->img_gu, x, T, hid / 8, d.books, L->cb0, L->side))) return rc;
    if ((rc = mark_side(L, L->ev_img))) return rc;
    if (shared && ((rc = shared_gateup(L, x, T, 0, d.shared_inter, L->side)) ||
                   (rc = shared_down(L, T, 0, L->nsh, true, L->sh_part, 0, hid, L->side))))
        return rc;
    if ((rc = mark_side(L, L->ev_shared))) return rc;

    // 1. router + exact top-k (+ shared-gate sigmoid)
    rc = router_launch(d.router, d.shared_gate_w ? d.shared_gate : nullptr, x, T, E, hid, K,
                       d.renorm, route_cfg(d), L->rparts, L->rpart, L->ticket, L->idx, L->w,
                       L->sg, st);
    if (rc) return rc;
    if ((rc = join_side(L->ev_img, st))) return rc;
    mark(L, 1, st);

    // 2. gate/up gather: groups (token, kind), K matrices each
    GatherArgs a = {};
    a.nv = hid / 8;
    a.nchunks = L->nch_gu;
    a.M = inter;
    a.qb_per_mat = 4 * ((inter + kBlk - 1) / kBlk);
    a.mpg = K;
    a.gpt = 2;
    a.K = K;
    a.n_groups = T * 2;
    a.total = (long long)a.n_groups * a.nchunks * a.mpg * a.qb_per_mat;
    a.partial = L->pgu;
    a.bank = d.bank;
    a.rec_bytes = d.rec_bytes;
    a.kind_off[0] = L->off[0];
    a.kind_off[1] = L->off[1];
    a.kind_off[2] = L->off[2];
    a.route_idx = L->idx;
    a.image = L->img_gu;
    a.err = L->err;
    if ((rc = gather_launch(a, L->tiled, st))) return rc;
    mark(L, 2, st);

    // 3. SwiGLU and the down tables
    cudaError_t e = launch_pdl(moe_mid_kernel, dim3(T * K * L->nch_d * kMidSplit),
                               dim3(kMidThreads), 0, st, (const float *)L->pgu, L->nch_gu,
                               (size_t)T * 2 * K * inter, (const int *)L->idx, d.bank,
                               d.rec_bytes, L->off[3], K, inter, d.books, L->cb0 + 6, L->nch_d,
                               L->img_d, (const int *)nullptr, 0);
    if (e != cudaSuccess) return cuda_fail(e, "moe_mid_kernel");
    count_launch();
    mark(L, 3, st);

    // 4. down gather: one group per route, its own tables
    GatherArgs b = a;
    b.nv = inter / 8;
    b.nchunks = L->nch_d;
    b.M = hid;
    b.qb_per_mat = 4 * ((hid + kBlk - 1) / kBlk);
    b.mpg = 1;
    b.gpt = K;
    b.n_groups = T * K;
    b.total = (long long)b.n_groups * b.nchunks * b.qb_per_mat;
    b.partial = L->pd;
    b.image = L->img_d;
    b.early = pdl_enabled() ? 1 : 0;  // the routing is three kernels back
    if ((rc = gather_launch(b, L->tiled, st))) return rc;
    mark(L, 4, st);

    // 5. the shared expert
    if ((rc = join_side(L->ev_shared, st))) return rc;
    mark(L, 5, st);

    // 6. combine in route order
    e = launch_pdl(moe_combine_kernel, dim3(T * cdiv(hid, kCombineCols)), dim3(256), 0, st,
                   (const float *)L->pd, L->nch_d, (size_t)T * K * hid, (const int *)L->idx,
                   (const float *)L->w, d.bank, d.rec_bytes, L->off[3], T, K, inter, hid,
                   (const float *)(shared ? L->sh_part : nullptr), 1,
                   (size_t)T * hid, (const float *)L->sg, residual, out);
    if (e != cudaSuccess) return cuda_fail(e, "moe_combine_kernel");
    count_launch();
    mark(L, 6, st);
    if (L->timing) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(st, &cs);
        if (cs != cudaStreamCaptureStatusActive) collect(L);
    }

    if (idx_out)
        cudaMemcpyAsync(idx_out, L->idx, (size_t)T * K * sizeof(int),
                        cudaMemcpyDeviceToDevice, st);
    if (w_out)
        cudaMemcpyAsync(w_out, L->w, (size_t)T * K * sizeof(float),
                        cudaMemcpyDeviceToDevice, st);
    return WARP_OK;
}

extern "C" int warp_moe_layer_forward(warp_moe_layer *L, const float *x, int T,
                                      const float *residual, float *out,
                                      int *idx_out, float *w_out, void *stream) {
    return forward_impl(L, x, T, residual, out, idx_out, w_out, stream);
}

// The block form: the norm into the layer's own buffer, then the layer with
// h as the residual.  (Forming RMSNorm(h) inside the router, table and
// shared-expert kernels instead measured slower: each then waits on its own
// reduction over h, and two of them sit on the critical path.)
extern "C" int warp_moe_block_forward(warp_moe_layer *L, const float *h, int T,
                                      const float *norm_w, float eps, float *out,
                                      int *idx_out, float *w_out, void *stream) {
    WARP_ARG(L && h && out && out != h && T >= 1 && T <= L->max_tokens,
             "moe_block_forward: bad arguments (out must be another buffer than h)");
    const int rc = warp_rmsnorm(h, norm_w, L->xn, T, L->d.hidden, eps, stream);
    if (rc) return rc;
    return forward_impl(L, L->xn, T, h, out, idx_out, w_out, stream);
}

extern "C" int warp_moe_layer_forward_ep(warp_moe_layer *L, const float *x, int T,
                                         float *slots, int *idx_out, float *w_out,
                                         void *stream) {
    WARP_ARG(L && x && slots && T >= 1 && T <= L->max_tokens,
             "moe_layer_forward_ep: bad arguments");
    const warp_moe_desc &d = L->d;
    cudaStream_t st = (cudaStream_t)stream;
    const int hid = d.hidden, inter = d.inter, E = d.n_experts, K = d.top_k;
    const int max_routes = L->max_tokens * K;
    int rc;
    mark(L, 0, st);
    const bool shared = d.shared_gate_w != nullptr;
    const int S = K + L->nsh;                     // slots per token
    // this rank's blocks of the shared expert: [b0, b1) of nsh, and the
    // gate/up rows [r0, r1) that feed them
    const int b0 = (int)((long long)L->nsh * L->ep_rank / L->ep_size);
    const int b1 = (int)((long long)L->nsh * (L->ep_rank + 1) / L->ep_size);
    const int r0 = shared ? (int)((long long)d.shared_inter * b0 / L->nsh) : 0;
    const int r1 = shared ? (int)((long long)d.shared_inter * b1 / L->nsh) : 0;

    // 0. side stream: the gate/up tables of every token, then this rank's
    // blocks of the shared expert straight into their slots; the routing of
    // every token (the same on every rank), this rank's work routes
    if ((rc = fork_side(L, st))) return rc;
    if ((rc = lut_images(L->img_gu, x, T, hid / 8, d.books, L->cb0, L->side))) return rc;
    if ((rc = mark_side(L, L->ev_img))) return rc;
    if (shared && b1 > b0 &&
        ((rc = shared_gateup(L, x, T, r0, r1, L->side)) ||
         (rc = shared_down(L, T, b0, b1, false, slots + (size_t)K * hid, hid,
                           (long long)S * hid, L->side))))
        return rc;
    if ((rc = mark_side(L, L->ev_shared))) return rc;
    rc = router_launch(d.router, d.shared_gate_w ? d.shared_gate : nullptr, x, T, E, hid, K,
                       d.renorm, route_cfg(d), L->rparts, L->rpart, L->ticket, L->idx, L->w,
                       L->sg, st);
    if (rc) return rc;
    ep_plan_kernel<<<1, kPlanThreads, 0, st>>>(L->idx, T * K, L->ep_rank, L->ep_size,
                                               L->ep_mode, L->plan, max_routes, L->inv);
    WARP_CHECK_LAUNCH("ep_plan_kernel");
    if ((rc = join_side(L->ev_img, st))) return rc;
    mark(L, 1, st);

    // 1. gate/up gather over the work routes: group 2r + kind, one matrix
    GatherArgs a = {};
    a.nv = hid / 8;
    a.nchunks = L->nch_gu;
    a.M = inter;
    a.qb_per_mat = 4 * ((inter + kBlk - 1) / kBlk);
    a.mpg = 1;
    a.gpt = 2;
    a.K = K;
    a.n_groups = max_routes * 2;
    a.total = (long long)a.n_groups * a.nchunks * a.qb_per_mat;
    a.partial = L->pgu;
    a.bank = d.bank;
    a.rec_bytes = d.rec_bytes;
    a.kind_off[0] = L->off[0];
    a.kind_off[1] = L->off[1];
    a.kind_off[2] = L->off[2];
    a.image = L->img_gu;
    a.err = L->err;
    a.plan = L->plan;
    a.max_routes = max_routes;
    if ((rc = gather_launch(a, L->tiled, st))) return rc;
    mark(L, 2, st);

    // 2. SwiGLU and the down tables of the work routes
    cudaError_t e = launch_pdl(moe_mid_kernel, dim3(max_routes * L->nch_d * kMidSplit),
                               dim3(kMidThreads), 0, st, (const float *)L->pgu, L->nch_gu,
                               (size_t)max_routes * 2 * inter, (const int *)L->idx, d.bank,
                               d.rec_bytes, L->off[3], K, inter, d.books, L->cb0 + 6, L->nch_d,
                               L->img_d, (const int *)L->plan, max_routes);
    if (e != cudaSuccess) return cuda_fail(e, "moe_mid_kernel");
    count_launch();
    mark(L, 3, st);

    // 3. down gather over the work routes
    GatherArgs b = a;
    b.nv = inter / 8;
    b.nchunks = L->nch_d;
    b.M = hid;
    b.qb_per_mat = 4 * ((hid + kBlk - 1) / kBlk);
    b.gpt = 1;
    b.n_groups = max_routes;
    b.total = (long long)b.n_groups * b.nchunks * b.qb_per_mat;
    b.partial = L->pd;
    b.image = L->img_d;
    b.early = 1;                  // the plan is three kernels back
    if ((rc = gather_launch(b, L->tiled, st))) return rc;
    mark(L, 4, st);

    // 4. the shared expert
    if ((rc = join_side(L->ev_shared, st))) return rc;
    mark(L, 5, st);

    // 5. the routed slots, zeros where another rank contributes
    const size_t n_slots = (size_t)T * S * hid;
    moe_slots_kernel<<<cdiv(n_slots, 256), 256, 0, st>>>(
        L->pd, L->nch_d, (size_t)max_routes * hid, L->plan, max_routes, L->inv, d.bank,
        d.rec_bytes, L->off[3], T, K, L->nsh, inter, hid, b0, b1, slots);
    WARP_CHECK_LAUNCH("moe_slots_kernel");
    mark(L, 6, st);
    if (L->timing) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(st, &cs);
        if (cs != cudaStreamCaptureStatusActive) collect(L);
    }
    if (idx_out)
        cudaMemcpyAsync(idx_out, L->idx, (size_t)T * K * sizeof(int),
                        cudaMemcpyDeviceToDevice, st);
    if (w_out)
        cudaMemcpyAsync(w_out, L->w, (size_t)T * K * sizeof(float),
                        cudaMemcpyDeviceToDevice, st);
    return WARP_OK;
}

extern "C" int warp_moe_layer_combine(warp_moe_layer *L, const float *slots, int T,
                                      const float *residual, float *out, void *stream) {
    WARP_ARG(L && slots && out && T >= 1 && T <= L->max_tokens,
             "moe_layer_combine: bad arguments");
    const warp_moe_desc &d = L->d;
    const size_t n = (size_t)T * d.hidden;
    moe_combine_slots_kernel<<<cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>(
        slots, L->w, T, d.top_k, d.top_k + L->nsh, d.hidden, L->nsh, L->sg, residual, out);
    WARP_CHECK_LAUNCH("moe_combine_slots_kernel");
    return WARP_OK;
}

extern "C" int warp_moe_layer_slots_per_token(warp_moe_layer *L) {
    if (!L) return WARP_E_ARG;
    return L->d.top_k + L->nsh;
}

extern "C" int warp_moe_layer_prefill(warp_moe_layer *L, const float *x, int T,
                                      const float *residual, float *out, int *idx_out,
                                      float *w_out, void *stream) {
    WARP_ARG(L && x && out && T >= 1, "moe_layer_prefill: bad arguments");
    WARP_ARG(L->pf_ws && T <= L->pf_tokens,
             "moe_layer_prefill: T exceeds the layer's prefill_tokens (%d)", L->pf_tokens);
    WARP_ARG(((uintptr_t)x & 15) == 0, "moe_layer_prefill: x must be 16-byte aligned");
    const warp_moe_desc &d = L->d;
    cudaStream_t st = (cudaStream_t)stream;
    const int hid = d.hidden, inter = d.inter, E = d.n_experts, K = d.top_k, R = T * K;
    const bool shared = d.shared_gate_w != nullptr;
    int rc;
    // phases (with timing on): router + grouping, gate/up GEMM, (none),
    // down GEMM, shared expert, combine
    mark(L, 0, st);

    // 1. routing of every token, 2. the routes grouped by expert
    rc = router_launch(d.router, shared ? d.shared_gate : nullptr, x, T, E, hid, K, d.renorm,
                       route_cfg(d), L->pf_parts, L->pf_logits, L->pf_ticket, L->pf_idx,
                       L->pf_w, L->pf_sg, st);
    if (rc) return rc;
    if ((rc = prefill_group(L->pf_idx, R, E, L->pf_counts, L->pf_offsets, L->pf_slot_route,
                            L->pf_items_buf, L->pf_items, st)))
        return rc;
    // the B operand of the gate/up GEMMs: x in fp16, once
    if ((rc = prefill_half(x, L->pf_xh, (size_t)T * hid, st))) return rc;
    mark(L, 1, st);

    // 3. routed gate + up with SwiGLU -> H [slot][inter] fp16
    PfGemm g = {};
    g.bank = d.bank;
    g.rec_bytes = d.rec_bytes;
    g.tiled = L->tiled ? 1 : 0;
    g.code_off[0] = L->off[0];
    g.code_off[1] = L->off[1];
    g.sc_off[0] = L->off[3];
    g.sc_off[1] = L->off[3] + 2 * inter;
    g.books[0] = d.books + (size_t)L->cb0 * kEnt * kVec;
    g.books[1] = d.books + (size_t)(L->cb0 + 3) * kEnt * kVec;
    g.M = inter;
    g.Kd = hid;
    g.Xh = L->pf_xh;
    g.slot_route = L->pf_slot_route;
    g.K = K;
    g.T = T;
    g.items = L->pf_items_buf;
    g.Hout = L->pf_h;
    g.slots = L->pf_slots;
    g.hid = hid;
    g.err = L->err;
    if ((rc = prefill_gemm(g, false, true, L->pf_items, st))) return rc;
    mark(L, 2, st);
    mark(L, 3, st);

    // 4. routed down -> slots (t, j)
    PfGemm h = g;
    h.code_off[0] = L->off[2];
    h.sc_off[0] = L->off[3] + 4 * inter;
    h.books[0] = d.books + (size_t)(L->cb0 + 6) * kEnt * kVec;
    h.M = hid;
    h.Kd = inter;
    h.Hin = L->pf_h;
    if ((rc = prefill_gemm(h, false, false, L->pf_items, st))) return rc;
    mark(L, 4, st);

    // 5. the shared expert over all tokens -> slots (t, K): Q4 on the
    // prefill GEMM; another format through the trunk matmul, 64 tokens a
    // launch ([gate; up], then down over silu(gate) * up)
    if (shared && d.shared_bits != 4) {
        const int si = d.shared_inter, grp = d.shared_group, bits = d.shared_bits;
        const int ng_h = (hid + grp - 1) / grp, ng_i = (si + grp - 1) / grp;
        const size_t rb_h = (size_t)ng_h * grp * bits / 8, rb_i = (size_t)ng_i * grp * bits / 8;
        for (int t0 = 0; t0 < T; t0 += kMvqMaxBatch) {
            const int n = T - t0 < kMvqMaxBatch ? T - t0 : kMvqMaxBatch;
            MvqArgs m = {};
            m.seg[0] = {(const uint8_t *)d.shared_gate_w, d.shared_gate_s, si, 0};
            m.seg[1] = {(const uint8_t *)d.shared_up_w, d.shared_up_s, si, si};
            m.nseg = 2;
            m.in = hid;
            m.group = grp;
            m.bits = bits;
            m.rowbytes = rb_h;
            m.batch = n;
            m.X = x + (size_t)t0 * hid;
            m.Y = L->pf_sq_y;
            m.y_stride = 2 * si;
            m.xf = L->pf_sq_xf;
            if ((rc = mvq_launch(m, st))) return rc;
            MvqArgs q = {};
            q.seg[0] = {(const uint8_t *)d.shared_down_w, d.shared_down_s, hid, 0};
            q.nseg = 1;
            q.in = si;
            q.group = grp;
            q.bits = bits;
            q.rowbytes = rb_i;
            q.batch = n;
            q.act_a = L->pf_sq_y;
            q.act_b = L->pf_sq_y + si;
            q.act_stride = 2 * si;
            q.Y = L->pf_slots + ((size_t)t0 * (K + 1) + K) * hid;
            q.y_stride = (long long)(K + 1) * hid;
            q.xf = L->pf_sq_xf;
            if ((rc = mvq_launch(q, st))) return rc;
        }
    } else if (shared) {
        const int si = d.shared_inter, grp = d.shared_group;
        PfGemm a = {};
        a.qw[0] = (const uint8_t *)d.shared_gate_w;
        a.qw[1] = (const uint8_t *)d.shared_up_w;
        a.qs[0] = d.shared_gate_s;
        a.qs[1] = d.shared_up_s;
        a.q_group = grp;
        a.q_rowbytes = (size_t)((hid + grp - 1) / grp) * grp / 2;
        a.M = si;
        a.Kd = hid;
        a.Xh = L->pf_xh;
        a.K = K;
        a.T = T;
        a.Hout = L->pf_hs;
        a.err = L->err;
        const int nt = (T + 127) / 128;
        if ((rc = prefill_gemm(a, true, true, nt, st))) return rc;
        PfGemm b = a;
        b.qw[0] = (const uint8_t *)d.shared_down_w;
        b.qs[0] = d.shared_down_s;
        b.q_rowbytes = (size_t)((si + grp - 1) / grp) * grp / 2;
        b.M = hid;
        b.Kd = si;
        b.Hin = L->pf_hs;
        b.slots = L->pf_slots;
        b.hid = hid;
        if ((rc = prefill_gemm(b, true, false, nt, st))) return rc;
    }
    mark(L, 5, st);

    // 6. combine in route order
    const size_t n = (size_t)T * hid;
    moe_combine_slots_kernel<<<cdiv(n, 256), 256, 0, st>>>(L->pf_slots, L->pf_w, T, K, K + 1,
                                                          hid, shared ? 1 : 0, L->pf_sg,
                                                          residual, out);
    WARP_CHECK_LAUNCH("moe_combine_slots_kernel");
    mark(L, 6, st);
    if (L->timing) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        cudaStreamIsCapturing(st, &cs);
        if (cs != cudaStreamCaptureStatusActive) collect(L);
    }
    if (idx_out)
        cudaMemcpyAsync(idx_out, L->pf_idx, (size_t)R * sizeof(int), cudaMemcpyDeviceToDevice, st);
    if (w_out)
        cudaMemcpyAsync(w_out, L->pf_w, (size_t)R * sizeof(float), cudaMemcpyDeviceToDevice, st);
    return WARP_OK;
}

// Device-side status of the layer's kernels (0 = fine).
extern "C" int warp_moe_layer_status(warp_moe_layer *L, void *stream) {
    if (!L) return WARP_E_ARG;
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, L->err, sizeof(int), cudaMemcpyDeviceToHost,
                                    (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_fail(e, "moe status");
    if (h & 2) {
        set_error("moe: a tensor-core kernel gave up waiting for its MMAs");
        return WARP_E_TIMEOUT;
    }
    if (h) {
        set_error("moe: gather kernel could not place its tables in shared memory");
        return WARP_E_CUDA;
    }
    return WARP_OK;
}

// Turn phase timing on (events recorded around every phase; each forward
// then synchronizes on its last event, so this is for measurement runs,
// never for graph capture) or off, clearing the totals.
extern "C" int warp_moe_layer_set_timing(warp_moe_layer *L, int on) {
    if (!L) return WARP_E_ARG;
    if (on && !L->timing) {
        for (int i = 0; i < 8; i++) {
            cudaError_t e = cudaEventCreate(&L->ev[i]);
            if (e != cudaSuccess) return cuda_fail(e, "timing events");
        }
    }
    if (!on && L->timing)
        for (int i = 0; i < 8; i++) cudaEventDestroy(L->ev[i]);
    L->timing = on != 0;
    for (int i = 0; i < 8; i++) L->phase_ms[i] = 0.0;
    L->phase_n = 0;
    return WARP_OK;
}

// Accumulated milliseconds per phase (router, gate/up gather, SwiGLU, down
// gather, shared expert, combine) into ms[6]; returns the forward count.
extern "C" int warp_moe_layer_timings(warp_moe_layer *L, double *ms) {
    if (!L || !ms) return WARP_E_ARG;
    for (int i = 0; i < PH_N; i++) ms[i] = L->phase_ms[i];
    return L->phase_n;
}

// After a replay of a graph captured with timing on: add the phase times of
// that replay to the totals (synchronizes on the layer's last event).
extern "C" int warp_moe_layer_collect(warp_moe_layer *L) {
    if (!L || !L->timing) return WARP_E_ARG;
    collect(L);
    return WARP_OK;
}
