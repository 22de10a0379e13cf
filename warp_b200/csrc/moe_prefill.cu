// moe_prefill.cu — grouped tensor-core GEMMs of the MoE layer for many
// tokens (the prefill path of moe_chunk, model.c:7110-7290, which routes all
// tokens, reads each distinct expert once and applies it to its tokens).
//
// Each CTA (16 warps) owns one n-tile (<= 128 tokens of one expert, or of the
// shared expert) and one 128-row tile of the weight matrix.  Per 128-wide K
// step the threads dequantize the weight rows into fp16 operand tiles (VQ3R:
// (C0 + C1) + C2 summed in fp16 from the container's fp16 codebooks — one
// rounding more than the fp32 sum of the bit-exact dequant, well inside the
// FFN tolerance; Q4: (n - 8) * group scale, rounded once) while the step's
// fp16 token rows stream into the stage with cp.async, and thread 0 issues
// the K = 16 MMAs of the step (two accumulators
// for the gate/up pair) and commits them to the stage's mbarrier; the other
// stage fills meanwhile.  Row scales of VQ3R
// matrices are applied to the fp32 accumulators in the epilogue, as vq_rows
// applies them (model.c:3974-3976).
#include "moe_prefill.cuh"
#include "umma.cuh"
#include "vq_gather.cuh"

namespace warp {

constexpr int kPfThreads = 512;
constexpr int kPfRows = 128;              // MMA M
constexpr int kPfTok = 128;               // max tokens per n-tile (MMA N)
constexpr int kPfK = 128;                 // K per pipeline step (16 vector positions)
constexpr int kPfKG = kPfK / 8;           // 16-byte k-groups per step
constexpr uint32_t kPfTile = kPfRows * kPfK * 2;   // one operand tile, 32 KiB

// ----------------------------------------------------------------- grouping

constexpr int kGroupThreads = 1024;

__global__ void __launch_bounds__(kGroupThreads)
prefill_group_kernel(const int *__restrict__ idx, int R, int E, int *__restrict__ counts,
                     int *__restrict__ offsets, int *__restrict__ slot_route,
                     int *__restrict__ items, int max_items) {
    __shared__ int cnt[384], off[385], fill[384];
    for (int e = threadIdx.x; e < E; e += kGroupThreads) { cnt[e] = 0; fill[e] = 0; }
    __syncthreads();
    for (int r = threadIdx.x; r < R; r += kGroupThreads) {
        const int e = idx[r];
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        off[0] = 0;
        for (int e = 0; e < E; e++) off[e + 1] = off[e] + cnt[e];
    }
    __syncthreads();
    // slot order inside an expert is irrelevant: each token is its own column
    for (int r = threadIdx.x; r < R; r += kGroupThreads) {
        const int e = idx[r];
        if (e >= 0 && e < E) slot_route[off[e] + atomicAdd(&fill[e], 1)] = r;
    }
    for (int e = threadIdx.x; e < E; e += kGroupThreads) {
        counts[e] = cnt[e];
        offsets[e] = off[e];
    }
    if (threadIdx.x == 0) {
        offsets[E] = off[E];
        int n = 0;
        for (int e = 0; e < E; e++)
            for (int s = 0; s < cnt[e]; s += kPfTok) {
                if (n < max_items) {
                    items[1 + 3 * n] = e;
                    items[2 + 3 * n] = off[e] + s;
                    items[3 + 3 * n] = min(kPfTok, cnt[e] - s);
                }
                n++;
            }
        items[0] = min(n, max_items);
    }
}

int prefill_group(const int *idx, int R, int E, int *counts, int *offsets, int *slot_route,
                  int *items, int max_items, cudaStream_t st) {
    WARP_ARG(E >= 1 && E <= 384 && R >= 1, "prefill: bad routing shape");
    prefill_group_kernel<<<1, kGroupThreads, 0, st>>>(idx, R, E, counts, offsets, slot_route,
                                                      items, max_items);
    WARP_CHECK_LAUNCH("prefill_group_kernel");
    return WARP_OK;
}

// ---------------------------------------------------------------- the GEMMs

__device__ __forceinline__ uint32_t h2pack(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
}

__device__ __forceinline__ uint32_t hadd2u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__global__ void prefill_half_kernel(const float4 *__restrict__ x, uint4 *__restrict__ xh,
                                    size_t n8) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    const float4 a = x[2 * i], b = x[2 * i + 1];
    xh[i] = make_uint4(h2pack(a.x, a.y), h2pack(a.z, a.w), h2pack(b.x, b.y), h2pack(b.z, b.w));
}

int prefill_half(const float *x, uint16_t *xh, size_t n, cudaStream_t st) {
    WARP_ARG(n % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)xh & 15) == 0,
             "prefill: fp16 conversion needs 8-element, 16-byte aligned rows");
    const size_t n8 = n / 8;
    if (n8 == 0) return WARP_OK;
    prefill_half_kernel<<<cdiv(n8, 256), 256, 0, st>>>((const float4 *)x, (uint4 *)xh, n8);
    WARP_CHECK_LAUNCH("prefill_half_kernel");
    return WARP_OK;
}

// 8 fp16 weights of row r, k-group kg of a Q4 matrix (rows `mat`, group
// scales qs): (nibble - 8) * scale, low nibble first (waste_mvq_rows_f32).
__device__ __forceinline__ uint4 q4_vector(const PfGemm &g, const uint8_t *mat,
                                           const uint16_t *qs, int r, int kg) {
    if (r >= g.M || kg * 8 >= g.Kd) return make_uint4(0u, 0u, 0u, 0u);
    const uint32_t w = *(const uint32_t *)(mat + (size_t)r * g.q_rowbytes + kg * 4);
    const int ng = (g.Kd + g.q_group - 1) / g.q_group;
    const float s = f16_to_f32(qs[(size_t)r * ng + (kg * 8) / g.q_group]);
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; j++) f[j] = (float)((int)((w >> (4 * j)) & 15u) - 8) * s;
    return make_uint4(h2pack(f[0], f[1]), h2pack(f[2], f[3]), h2pack(f[4], f[5]),
                      h2pack(f[6], f[7]));
}

// VQ3R weights are dequantized per unit of (one vector position, one 16-row
// quarter): the unit's 48 code bytes (16 rows x 3 stages) are three aligned
// 16-byte pieces in both index layouts.  A thread decodes S of the 16 row
// slots and reads only their 3S/4 code words, one K step ahead of use.
struct VqUnit {
    const uint8_t *src;        // piece 0, or NULL: the unit is outside the matrix
    uint32_t pstride;          // bytes between the pieces
    int xr;                    // tile layout: slot i holds row 16q + (i ^ xr)
};

__device__ __forceinline__ VqUnit vq_unit(const PfGemm &g, const uint8_t *mat, int m0, int qq,
                                          int v) {
    VqUnit u;
    u.src = nullptr;
    u.pstride = 16;
    u.xr = 0;
    const int nv = g.Kd / kVec;
    const int r0 = m0 + 16 * qq;
    if (v >= nv || r0 >= ((g.M + 63) & ~63)) return u;
    const int rb = r0 >> 6, q = (r0 >> 4) & 3;
    if (g.tiled) {
        const int c = v >> 5, p = v & 31;
        const int npos = min(kChunk, nv - c * kChunk);
        u.src = mat + ((size_t)rb * nv + c * kChunk) * (kBlk * kSt) + q * (npos * 48) + p * 16;
        u.pstride = npos * 16;
        u.xr = p & 15;
    } else {
        u.src = mat + (((size_t)rb * nv + v) * kBlk + 16 * q) * kSt;
    }
    return u;
}

// Words NW*h .. NW*h+NW-1 of the unit's 48 bytes: the codes of row slots
// S*h .. S*h+S-1.
template <int S>
__device__ __forceinline__ void vq_unit_load(const VqUnit &u, int h, uint32_t (&w)[3 * S / 4]) {
    constexpr int NW = 3 * S / 4;
#pragma unroll
    for (int k = 0; k < NW; k++) {
        const int word = NW * h + k;
        w[k] = u.src ? __ldg((const uint32_t *)(u.src + (word >> 2) * u.pstride + (word & 3) * 4))
                     : 0u;
    }
}

// Codebooks in shared memory as fp16, every entry stored kRep times side by
// side: entry e (stage-major, s*256 + code) copy k at e*kRep*16 + k*16.  A
// lane reads copy (lane & 7), so the eight lanes of a quarter-warp's 16-byte
// loads land on eight different bank groups whatever their codes are: the
// random codebook gathers run without bank conflicts.
constexpr int kRep = 8;
constexpr uint32_t kPfBooksRep = kSt * kEnt * kRep * 16;    // 96 KiB per matrix

__device__ __forceinline__ void fill_books(uint8_t *sb, const float *books, int tid) {
    for (int i = tid; i < kSt * kEnt * kRep; i += kPfThreads) {
        const float4 *e = (const float4 *)(books + (size_t)(i / kRep) * kVec);
        const float4 lo = e[0], hi = e[1];
        *(uint4 *)(sb + (size_t)i * 16) = make_uint4(h2pack(lo.x, lo.y), h2pack(lo.z, lo.w),
                                                     h2pack(hi.x, hi.y), h2pack(hi.z, hi.w));
    }
}

// Decode row slots S*h .. S*h+S-1 of a unit into its k-group column of the A
// tile (Akg = tile + kg * 128 * 16): row = 16*qq + (slot ^ xr).  sbr: this
// lane's copy of the replicated fp16 codebooks.  (C0 + C1) + C2 in fp16.
template <int S>
__device__ __forceinline__ void vq_unit_decode(const uint32_t (&w)[3 * S / 4], const VqUnit &u,
                                               int h, int qq, int rows_left, const uint8_t *sbr,
                                               uint8_t *Akg) {
#pragma unroll
    for (int ii = 0; ii < S; ii++) {
        const int row = 16 * qq + ((S * h + ii) ^ u.xr);
        uint4 hv = make_uint4(0u, 0u, 0u, 0u);
        if (u.src && row < rows_left) {
            const uint32_t c0 = (w[(3 * ii) >> 2] >> (((3 * ii) & 3) * 8)) & 255u;
            const uint32_t c1 = (w[(3 * ii + 1) >> 2] >> (((3 * ii + 1) & 3) * 8)) & 255u;
            const uint32_t c2 = (w[(3 * ii + 2) >> 2] >> (((3 * ii + 2) & 3) * 8)) & 255u;
            const uint4 e0 = *(const uint4 *)(sbr + (0 * kEnt + c0) * (kRep * 16));
            const uint4 e1 = *(const uint4 *)(sbr + (1 * kEnt + c1) * (kRep * 16));
            const uint4 e2 = *(const uint4 *)(sbr + (2 * kEnt + c2) * (kRep * 16));
            hv = make_uint4(hadd2u(hadd2u(e0.x, e1.x), e2.x), hadd2u(hadd2u(e0.y, e1.y), e2.y),
                            hadd2u(hadd2u(e0.z, e1.z), e2.z), hadd2u(hadd2u(e0.w, e1.w), e2.w));
        }
        *(uint4 *)(Akg + row * 16) = hv;
    }
}

// Shared memory of a launch form.  VQ3R forms hold one matrix's replicated
// codebooks; the VQ3R gate/up pair runs its two matrices one after the
// other (gate over all K, then up, into the pair's two accumulators), so a
// step decodes one A tile.  The Q4 pair decodes both A tiles per step.
template <bool Q4, bool PAIR>
struct PfLayout {
    static constexpr bool SEQ = !Q4 && PAIR;     // one matrix per pass
    static constexpr int NA = PAIR ? 2 : 1;      // accumulators
    static constexpr int NM = (Q4 && PAIR) ? 2 : 1;   // A tiles per step
    static constexpr uint32_t books = 0;
    static constexpr uint32_t stage0 = Q4 ? 0 : kPfBooksRep;
    static constexpr uint32_t stage_bytes = (NM + 1) * kPfTile;
    static constexpr uint32_t bar = stage0 + 2 * stage_bytes;
    static constexpr uint32_t tslot = bar + 16;
    static constexpr int smem = tslot + 16 + 1024;
    static constexpr uint32_t tcols = PAIR ? 256 : 128;
};

template <bool Q4, bool PAIR, bool BX>
__global__ void __launch_bounds__(kPfThreads, 1)
pf_gemm_kernel(const PfGemm g) {
    using Lay = PfLayout<Q4, PAIR>;
    extern __shared__ uint8_t smem_raw[];
    // the work item
    int e = -1, s0, n;
    if (g.items) {
        if ((int)blockIdx.y >= g.items[0]) return;
        e = g.items[1 + 3 * blockIdx.y];
        s0 = g.items[2 + 3 * blockIdx.y];
        n = g.items[3 + 3 * blockIdx.y];
    } else {
        s0 = blockIdx.y * kPfTok;
        n = min(kPfTok, g.T - s0);
    }
    const int m0 = blockIdx.x * kPfRows;
    if (n <= 0 || m0 >= g.M) return;
    const int Nt = (n + 15) & ~15;

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sp = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const uint8_t *mat0 = g.qw[0], *mat1 = g.qw[PAIR ? 1 : 0];
    const uint16_t *qs0 = g.qs[0], *qs1 = g.qs[PAIR ? 1 : 0];
    if (!Q4) {
        const uint8_t *rec = g.bank + (size_t)e * g.rec_bytes;
        mat0 = rec + g.code_off[0];
        mat1 = rec + g.code_off[PAIR ? 1 : 0];
        fill_books(sp + Lay::books, g.books[0], tid);
    }
    const uint32_t bar0 = base + Lay::bar, bar1 = bar0 + 8;
    if (tid == 0) {
        umma::mbar_init(bar0, 1);
        umma::mbar_init(bar1, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) umma::tmem_alloc(base + Lay::tslot, Lay::tcols);
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = *(volatile uint32_t *)(sp + Lay::tslot);
    const uint32_t idesc = umma::idesc_f16(kPfRows, Nt);

    const int ksteps = (g.Kd + kPfK - 1) / kPfK;
    const int nsteps = Lay::SEQ ? 2 * ksteps : ksteps;
    // VQ3R units of this thread: matrix um, position p16 of each K step,
    // quarter qq of the tile, part uh of the quarter's 16 row slots
    constexpr int TPM = kPfThreads / Lay::NM;            // threads per A tile
    constexpr int S = 16 * (kPfKG * 8) / TPM;            // row slots per thread
    constexpr int NW = 3 * S / 4;
    const int um = tid / TPM, urem = tid % TPM;
    const int p16 = urem & 15, qq = (urem >> 4) & 7, uh = urem >> 7;
    const uint8_t *sbr = sp + Lay::books + (lane & (kRep - 1)) * 16;
    uint32_t wn[NW];
    VqUnit un;
    if (!Q4) {
        un = vq_unit(g, um ? mat1 : mat0, m0, qq, p16);
        vq_unit_load<S>(un, uh, wn);
    }
    // B pieces of this thread (16 bytes: one token row, one k-group), the
    // same every step: piece pc = tid + j*512 holds row pc % Nt, k-group
    // pc / Nt; rows >= n are zero
    constexpr int kBP = kPfTok * kPfKG / kPfThreads;
    const uint16_t *bsrc[kBP];
    uint32_t bdst[kBP];
    int bkg[kBP];
#pragma unroll
    for (int j = 0; j < kBP; j++) {
        const int pc = tid + j * kPfThreads;
        bsrc[j] = nullptr;
        bdst[j] = ~0u;
        bkg[j] = 0;
        if (pc < Nt * kPfKG) {
            const int row = pc % Nt, kg = pc / Nt;
            bdst[j] = (uint32_t)(kg * (Nt * 16) + row * 16);
            bkg[j] = kg;
            if (row < n) {
                const int slot = s0 + row;
                const int t = BX ? (g.slot_route ? g.slot_route[slot] / g.K : slot) : slot;
                bsrc[j] = (BX ? g.Xh : g.Hin) + (size_t)t * g.Kd + kg * 8;
            }
        }
    }
    uint32_t ph0 = 0u, ph1 = 0u;
    bool ok = true;
    int issued = 0;
    for (int ks = 0; ks < nsteps; ks++) {
        const int s = ks & 1;
        if (ks >= 2) {
            const bool w = umma::mbar_wait(s ? bar1 : bar0, s ? ph1 : ph0, umma::kWaitLimit);
            if (s) ph1 ^= 1u; else ph0 ^= 1u;
            ok = __syncthreads_and(w);
            if (!ok) break;
        }
        // the pass (matrix) and K step of this step
        const int mi = Lay::SEQ ? (ks >= ksteps ? 1 : 0) : 0;
        const int kl = ks - mi * ksteps;
        if (Lay::SEQ && ks == ksteps) {
            // the up pass: every thread is done with the gate codebooks
            __syncthreads();
            fill_books(sp + Lay::books, g.books[1], tid);
            __syncthreads();
        }
        uint8_t *st = sp + Lay::stage0 + s * Lay::stage_bytes;
        // B tile: the step's token rows start streaming in first
        {
            uint8_t *Bp = st + Lay::NM * kPfTile;
            const uint32_t Bs = smem_u32(Bp);
#pragma unroll
            for (int j = 0; j < kBP; j++) {
                if (bdst[j] == ~0u) continue;
                if (bsrc[j] && kl * kPfK + bkg[j] * 8 < g.Kd)
                    cp_async16(Bs + bdst[j], bsrc[j] + (size_t)kl * kPfK);
                else
                    *(uint4 *)(Bp + bdst[j]) = make_uint4(0u, 0u, 0u, 0u);
            }
            cp_async_commit();
        }
        if (!Q4) {
            // VQ3R: the unit loaded one step ahead; the next step's words
            // are requested before this step's are decoded
            uint32_t wc[NW];
#pragma unroll
            for (int k = 0; k < NW; k++) wc[k] = wn[k];
            const VqUnit uc = un;
            if (ks + 1 < nsteps) {
                const int nx = ks + 1;
                const int nmi = Lay::SEQ ? (nx >= ksteps ? 1 : 0) : um;
                const int nkl = Lay::SEQ ? nx - (nx >= ksteps ? ksteps : 0) : nx;
                un = vq_unit(g, nmi ? mat1 : mat0, m0, qq, nkl * kPfKG + p16);
                vq_unit_load<S>(un, uh, wn);
            }
            vq_unit_decode<S>(wc, uc, uh, qq, g.M - m0, sbr,
                              st + um * kPfTile + p16 * (kPfRows * 16));
        } else {
            // Q4: TPM threads per matrix over 128 rows x 16 k-groups
            constexpr int KPT = kPfRows * kPfKG / TPM;   // k-groups per thread
            const int r = urem / (kPfKG / KPT), kq = urem % (kPfKG / KPT);
#pragma unroll 4
            for (int j = kq * KPT; j < kq * KPT + KPT; j++)
                *(uint4 *)(st + um * kPfTile + j * (kPfRows * 16) + r * 16) =
                    q4_vector(g, um ? mat1 : mat0, um ? qs1 : qs0, m0 + r, kl * kPfKG + j);
        }
        cp_async_wait<0>();                              // this thread's B pieces
        umma::fence_smem_async();
        __syncthreads();
        if (tid == 0) {
            umma::fence_after();
            const uint32_t S0 = base + Lay::stage0 + s * Lay::stage_bytes;
            const uint32_t B = S0 + Lay::NM * kPfTile;
#pragma unroll
            for (int kk = 0; kk < kPfKG / 2; kk++) {
                const uint64_t bd = umma::desc(B + 2 * kk * (Nt * 16), Nt * 16, 128);
                if (Lay::SEQ) {
                    umma::mma_f16(tmem + mi * 128,
                                  umma::desc(S0 + 2 * kk * (kPfRows * 16), kPfRows * 16, 128),
                                  bd, idesc, kl > 0 || kk > 0);
                } else {
#pragma unroll
                    for (int m = 0; m < Lay::NA; m++)
                        umma::mma_f16(tmem + m * 128,
                                      umma::desc(S0 + m * kPfTile + 2 * kk * (kPfRows * 16),
                                                 kPfRows * 16, 128),
                                      bd, idesc, ks > 0 || kk > 0);
                }
            }
            umma::commit(s ? bar1 : bar0);
        }
        issued = ks + 1;
    }
    bool done = true;
    if (issued > 0) {
        const int s = (issued - 1) & 1;
        done = umma::mbar_wait(s ? bar1 : bar0, s ? ph1 : ph0, umma::kWaitLimit);
    }
    done = __syncthreads_and(done);
    if (!ok || !done) {
        if (tid == 0) atomicOr(g.err, 2);
    } else {
        umma::fence_after();
        // warp w reads TMEM lanes 32*(w & 3) + lane; the four warps of each
        // lane quarter split the 16-column chunks round robin
        const int row = m0 + (warp & 3) * 32 + lane;
        const bool rok = row < g.M;
        float sc0 = 1.0f, sc1 = 1.0f;
        if (!Q4 && rok) {
            const uint8_t *rec = g.bank + (size_t)e * g.rec_bytes;
            sc0 = f16_to_f32(((const uint16_t *)(rec + g.sc_off[0]))[row]);
            if (PAIR) sc1 = f16_to_f32(((const uint16_t *)(rec + g.sc_off[1]))[row]);
        }
        const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        for (int c0 = (warp >> 2) * 16; c0 < Nt; c0 += 16 * (kPfThreads / 128)) {
            float d0[16];
            umma::tmem_ld16(lane_addr + (uint32_t)c0, d0);
            if (PAIR) {
                float d1[16];
                umma::tmem_ld16(lane_addr + 128u + (uint32_t)c0, d1);
                if (rok) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        if (c0 + j < n) {
                            const float gv = d0[j] * sc0, uv = d1[j] * sc1;
                            const float hv = (gv / (1.0f + expf(-gv))) * uv;
                            g.Hout[(size_t)(s0 + c0 + j) * g.M + row] =
                                __half_as_ushort(__float2half_rn(hv));
                        }
                    }
                }
            } else if (rok) {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (c0 + j < n) {
                        const int slot = s0 + c0 + j;
                        int t, jj;
                        if (g.slot_route) {
                            const int route = g.slot_route[slot];
                            t = route / g.K;
                            jj = route % g.K;
                        } else {
                            t = slot;
                            jj = g.K;
                        }
                        g.slots[((size_t)t * (g.K + 1) + jj) * g.hid + row] = d0[j] * sc0;
                    }
                }
            }
        }
    }
    umma::fence_before();
    __syncthreads();
    if (warp == 0) {
        umma::fence_after();
        umma::tmem_free(tmem, Lay::tcols);
    }
}

template <bool Q4, bool PAIR, bool BX>
static int launch_pf(const PfGemm &g, int grid_items, cudaStream_t st) {
    using Lay = PfLayout<Q4, PAIR>;
    static_assert(Lay::smem <= 227 * 1024, "prefill GEMM shared memory");
    auto fn = pf_gemm_kernel<Q4, PAIR, BX>;
    static bool attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr[dev]) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Lay::smem);
        if (e != cudaSuccess) return cuda_fail(e, "prefill gemm smem attribute");
        attr[dev] = true;
    }
    dim3 grid(cdiv(g.M, kPfRows), grid_items);
    fn<<<grid, kPfThreads, Lay::smem, st>>>(g);
    WARP_CHECK_LAUNCH("pf_gemm_kernel");
    return WARP_OK;
}

int prefill_gemm(const PfGemm &g, bool q4, bool pair, int grid_items, cudaStream_t st) {
    WARP_ARG(g.Kd % 8 == 0 && g.M >= 1 && grid_items >= 1, "prefill gemm: bad shape");
    if (grid_items > 65535) {
        set_error("prefill gemm: %d work items exceed one launch", grid_items);
        return WARP_E_ARG;
    }
    if (!q4 && pair) return launch_pf<false, true, true>(g, grid_items, st);
    if (!q4 && !pair) return launch_pf<false, false, false>(g, grid_items, st);
    if (q4 && pair) return launch_pf<true, true, true>(g, grid_items, st);
    return launch_pf<true, false, false>(g, grid_items, st);
}

}  // namespace warp
