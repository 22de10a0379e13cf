// mvq_umma.cu — the batched trunk matmul on the tensor cores (tcgen05), for
// 2..64 tokens: Y[t][o] = sum_g f16(ws[o][g]) * sum_{k in g} q(o, k) x[t][k],
// the arithmetic of waste_matmul_t / mmq_rows (model.c:6964-7028) up to fp32
// rounding.
//
//  * A = the weights as exact fp16 integers (Q4: nibble - 8, Q8: int8), 128
//    rows per CTA, one per tensor-memory lane of the accumulator;
//  * B = the tokens, each scaled by a power of two (its largest |x| into
//    [2^14, 2^15)) and split into fp16 hi + lo (about 22 significant bits
//    relative to that value): an MMA pair per 16 k adds q*hi and q*lo into
//    the same fp32 accumulator, and the output is scaled back exactly;
//  * one accumulator per scale group (32 k for g32, the CTA's whole k range
//    for a per-row Q8 scale) in one of NBUF rotating tensor-memory buffers;
//    B holds the tokens' hi rows and then their lo rows, so one MMA of
//    N = 2 NP per 16 k makes both products; the epilogue warps (thread =
//    row) read a finished accumulator back with tcgen05.ld and add
//    scale * (hi + lo) into registers in group order, so the per-group
//    scale stays an exact fp32 multiply (a scale folded into fp16 weights
//    would round).
// Roles (warp-specialised; measured, one thread issues a tcgen05.mma in
// about 60-90 cycles, so issuing must not wait on the conversion):
//  * warps 0-3, the epilogue (warp w reads lanes 32w..32w+31);
//  * warps 4-7, the converters: thread p owns row p, streams its raw bytes
//    and its share of the B tiles with cp.async kUPD stages ahead into
//    kUStg stage buffers, converts its row into the fp16 A tile (two
//    buffers) and, through thread 128, signals aready;
//  * warp 8, lane 0: the MMA issuer, with descriptors precomputed.
// Mbarriers: aready[i] (A and B of a stage in shared memory), full[b] (a
// group's MMAs done), empty[b] (the epilogue read buffer b), afree[i] /
// bfree[s] (the MMAs that read an A / stage buffer done; a refill waits for
// those of two stages back).  Every wait is bounded; a wait that gives up
// sets err and the CTA drains and returns.
// When the 128-row tiles alone do not fill the GPU, K is split over S CTAs
// per tile and mvq_umma_reduce_kernel adds the splits' partials in order.
#include "common.cuh"
#include "mvq.cuh"
#include "umma.cuh"

namespace warp {

constexpr int kURows = 128;        // rows per CTA (accumulator lanes)
constexpr int kUG = 2;             // 32-k blocks per stage
constexpr int kUStg = 4;           // stage buffers (raw weights + B tiles)
constexpr int kUPD = 2;            // stages loaded ahead: a refill waits for the MMAs of two stages back
constexpr int kUThreads = 288;     // 4 epilogue warps, 4 converter warps, 1 MMA warp

template <int BITS, int NP>
struct ULay {
    static constexpr int CPS = NP <= 32 ? 2 : 1;           // CTAs per SM
    static constexpr int RB = BITS == 4 ? 16 : 32;         // raw bytes per block per row
    static constexpr int PPR = kUG * RB / 16;              // 16-byte pieces per row
    static constexpr int RAWS = kUG * RB;                  // raw row stride
    // piece j of row r sits at slot j ^ ((r >> RSH) & (PPR - 1)): the rows
    // a quarter-warp converts read eight different bank quads
    static constexpr int RSH = RAWS == 32 ? 2 : 1;
    static constexpr int RAWB = kURows * RAWS;
    static constexpr int BTB = kUG * 128 * NP;             // B bytes per stage (hi and lo rows)
    static constexpr int ATB = kUG * kURows * 64;          // A bytes per buffer
    static constexpr int tcols = 512 / CPS;                // tensor memory per CTA
    static constexpr int NBUF = tcols / (2 * NP);          // accumulators of 2 NP columns
    static constexpr int raw = 0;
    static constexpr int btile = raw + kUStg * RAWB;
    static constexpr int atile = btile + kUStg * BTB;
    static constexpr int bars = atile + 2 * ATB;           // 8-byte mbarriers
    static constexpr int nbars = 2 * NBUF + 4 + kUStg;
    static constexpr int tslot = bars + 8 * nbars;
    static constexpr int used = tslot + 16 + 1024;         // + the 1 KiB alignment slack
    // one CTA per SM for the wide cases: ask for more than half the SM
    static constexpr int bytes = CPS == 1 && used < 120 * 1024 ? 120 * 1024 : used;
    static_assert(used <= (CPS == 2 ? 110 : 220) * 1024, "shared memory per CTA");
};

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
// The same, asking L2 to fetch the whole 256-byte block around src: a
// converter stage reads only 16-32 bytes of each of 128 rows, and the next
// stages read the bytes after them, which are then in L2 instead of another
// short DRAM access per row.
__device__ __forceinline__ void cp_async16_zfill_l2(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;"
                 ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, float *v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void producers_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Raw block of one row (its 16-byte pieces w0, w1) -> four 16-byte fp16
// k-groups of eight weights in k order (A layout: k-group kg of the block
// at a + kg * 2048, a = the row's 16 bytes).
template <int BITS>
__device__ __forceinline__ void convert_block(const uint4 w0, const uint4 w1, uint8_t *a) {
    if (BITS == 4) {
        const uint32_t ws[4] = {w0.x, w0.y, w0.z, w0.w};
#pragma unroll
        for (int kg = 0; kg < 4; kg++) {
            // byte m of word kg holds k = 8kg + 2m (low nibble), 8kg + 2m + 1
            const uint32_t lo = ws[kg] & 0x0F0F0F0Fu, hi = (ws[kg] >> 4) & 0x0F0F0F0Fu;
            uint32_t p[4];
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const uint32_t sel = (uint32_t)m | ((uint32_t)(4 + m) << 8);
                const uint32_t v = (prmt(lo, hi, sel) & 0x00FF00FFu) | 0x64006400u;
                p[m] = hsub2u(v, 0x64086408u);                 // (1024 + n) - 1032
            }
            *(uint4 *)(a + kg * 2048) = make_uint4(p[0], p[1], p[2], p[3]);
        }
    } else {
        const uint32_t ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int kg = 0; kg < 4; kg++) {
            uint32_t p[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t x = ws[2 * kg + h] ^ 0x80808080u;      // b + 128
                p[2 * h] = hsub2u(prmt(x, 0x64646464u, 0x4140u), 0x64806480u);
                p[2 * h + 1] = hsub2u(prmt(x, 0x64646464u, 0x4342u), 0x64806480u);
            }
            *(uint4 *)(a + kg * 2048) = make_uint4(p[0], p[1], p[2], p[3]);
        }
    }
}

// B tiles: bprep[kb][kg][2 NP][8 halves], rows 0..NP-1 the tokens' hi
// parts and NP..2NP-1 their lo parts, each 16 bytes apart (the no-swizzle
// K-major layout), and
// tscale[t] = the power of two that undoes the token's scaling.  CTA
// (t, c) of NP x gridDim.y finds token t's largest |x| (every CTA of the
// token reads the whole row, from L2) and converts the c-th share of its
// k-groups; rows >= batch are zero.
__global__ void __launch_bounds__(256)
mvq_umma_prep_kernel(const MvqArgs a, uint8_t *__restrict__ bprep, float *__restrict__ tscale,
                     int nkb, int NP) {
    __shared__ float red[8];
    const int t = blockIdx.x;
    const int u0 = (int)((long long)nkb * 4 * blockIdx.y / gridDim.y);
    const int u1 = (int)((long long)nkb * 4 * (blockIdx.y + 1) / gridDim.y);
    const bool live = t < a.batch;
    float mx = 0.0f;
    if (live)
        for (int k = threadIdx.x; k < a.in; k += 256) mx = fmaxf(mx, fabsf(x_at(a, t, k)));
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, m));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
    int E = 0;
    if (mx > 0.0f) frexpf(mx, &E);                       // mx = m * 2^E, m in [0.5, 1)
    const int up = mx > 0.0f ? 15 - E : 0;
    if (live && threadIdx.x == 0 && blockIdx.y == 0) tscale[t] = ldexpf(1.0f, -up);
    for (int u = u0 + threadIdx.x; u < u1; u += 256) {
        const int kb = u >> 2, kg = u & 3;
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float v[2] = {0.0f, 0.0f};
            if (live)
#pragma unroll
                for (int i = 0; i < 2; i++) v[i] = ldexpf(x_at(a, t, kb * 32 + kg * 8 + 2 * j + i), up);
            const __half h0 = __float2half_rn(v[0]), h1 = __float2half_rn(v[1]);
            const __half l0 = __float2half_rn(v[0] - __half2float(h0));
            const __half l1 = __float2half_rn(v[1] - __half2float(h1));
            h[j] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            l[j] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        uint8_t *base = bprep + (size_t)kb * (128 * NP) + (size_t)kg * (32 * NP) + (size_t)t * 16;
        *(uint4 *)base = make_uint4(h[0], h[1], h[2], h[3]);
        *(uint4 *)(base + 16 * NP) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// Row R of the (one or two segment) weight list.
__device__ __forceinline__ const uint8_t *urow(const MvqArgs &a, int R, const uint16_t **ws,
                                               int *yo) {
    const bool s1 = a.nseg > 1 && R >= a.seg[0].rows;
    const MvqSeg &sg = s1 ? a.seg[1] : a.seg[0];
    const int r = s1 ? R - a.seg[0].rows : R;
    *ws = sg.ws + (size_t)r * a.ng;
    *yo = sg.y_off + r;
    return sg.W + (size_t)r * a.rowbytes;
}

template <int BITS, int NPB>
__global__ void __launch_bounds__(kUThreads, ULay<BITS, 16 * NPB>::CPS)
mvq_umma_kernel(const MvqArgs a, const uint8_t *__restrict__ bprep,
                const float *__restrict__ tscale, float *__restrict__ part, int nkb, int S,
                int *__restrict__ err) {
    constexpr int NP = 16 * NPB;
    using Lay = ULay<BITS, NP>;
    constexpr int NBUF = Lay::NBUF;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ volatile int s_abort;         // written by any role that gives up
    __shared__ volatile int s_stop;          // the converters' copy, taken before a barrier
    const uint32_t sraw = smem_u32(smem_raw);
    const uint32_t base = (sraw + 1023u) & ~1023u;
    uint8_t *sp = smem_raw + (base - sraw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x / S, split = blockIdx.x % S;
    const int r0 = tile * kURows;
    const int kb0 = (int)((long long)nkb * split / S), kb1 = (int)((long long)nkb * (split + 1) / S);
    const int nst = (kb1 - kb0 + kUG - 1) / kUG;
    const int gpb = a.group >> 5;                       // 32-k blocks per scale group
    const int g0 = kb0 / gpb;
    const int nseg = (kb1 - 1) / gpb - g0 + 1;
    const uint32_t full = base + Lay::bars, empty = full + 8 * NBUF;
    const uint32_t aready = empty + 8 * NBUF, afree = aready + 16, bfree = afree + 16;
    if (tid == 0) {
        for (int b = 0; b < NBUF; b++) {
            umma::mbar_init(full + 8 * b, 1);
            umma::mbar_init(empty + 8 * b, 4);
        }
        for (int i = 0; i < 2; i++) {
            umma::mbar_init(aready + 8 * i, 1);
            umma::mbar_init(afree + 8 * i, 1);
        }
        for (int q = 0; q < kUStg; q++) umma::mbar_init(bfree + 8 * q, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_abort = 0;
        s_stop = 0;
    }
    if (warp == 0) umma::tmem_alloc(base + Lay::tslot, Lay::tcols);
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    const uint32_t tmem = *(volatile uint32_t *)(sp + Lay::tslot);

    if (warp < 4) {
        // ---- epilogue: thread = row; group g's accumulator holds the hi
        // and lo products in columns [0, NP) and [NP, 2 NP)
        const int R = r0 + tid;
        const bool rok = R < a.total_rows;
        const uint16_t *wsr = nullptr;
        int yo = 0;
        if (rok) urow(a, R, &wsr, &yo);
        float y[NP];
#pragma unroll
        for (int j = 0; j < NP; j++) y[j] = 0.0f;
        const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
        constexpr int CH = NP <= 32 ? NPB : 1;             // 16-column pairs per wait
        bool ok = true;
        float sc = rok ? f16_to_f32(wsr[g0]) : 0.0f;
        int b = 0;
        uint32_t ph = 0;
        for (int si = 0; si < nseg; si++) {
            const float scn = (rok && si + 1 < nseg) ? f16_to_f32(wsr[g0 + si + 1]) : 0.0f;
            const bool w = umma::mbar_wait(full + 8 * b, ph, umma::kWaitLimit);
            if (!__all_sync(0xffffffffu, w)) {
                if (lane == 0) atomicOr(err, 4);
                s_abort = 1;
                ok = false;
                break;
            }
            umma::fence_after();
            const uint32_t col = lane_addr + (uint32_t)(b * 2 * NP);
#pragma unroll
            for (int c0 = 0; c0 < NPB; c0 += CH) {
                float dh[16 * CH], dl[16 * CH];
#pragma unroll
                for (int c = 0; c < CH; c++) {
                    tmem_ld16_nowait(col + (uint32_t)((c0 + c) * 16), dh + 16 * c);
                    tmem_ld16_nowait(col + (uint32_t)(NP + (c0 + c) * 16), dl + 16 * c);
                }
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16 * CH; j++)
                    y[c0 * 16 + j] = __fmaf_rn(sc, __fadd_rn(dh[j], dl[j]), y[c0 * 16 + j]);
            }
            umma::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * b);
            sc = scn;
            if (++b == NBUF) { b = 0; ph ^= 1u; }
        }
        if (ok && rok) {
#pragma unroll
            for (int t = 0; t < NP; t++) {
                if (t >= a.batch) break;
                const float v = __fmul_rn(y[t], tscale[t]);
                if (S == 1) a.Y[(size_t)t * a.y_stride + yo] = v;
                else part[((size_t)split * a.batch + t) * a.total_rows + R] = v;
            }
        }
    } else if (warp < 8) {
        // ---- converters: thread p = row p; stage st's raw rows and B tiles
        // come in kUPD stages ahead, the row is converted into A, and p == 0
        // tells the MMA warp (aready) and waits for buffers to free up
        const int p = tid - 128;
        uint8_t *rawb = sp + Lay::raw, *atb = sp + Lay::atile;
        auto issue_stage = [&](int st) {
            if (st >= nst) {                               // past the end: an empty group
                cp_async_commit();
                return;
            }
            const int buf = st % kUStg;
            constexpr int PPR = Lay::PPR;
            for (int i = p; i < kURows * PPR; i += 128) {
                const int row = i / PPR, pc = i % PPR;
                const int kbl = pc / (Lay::RB / 16), sub = pc % (Lay::RB / 16);
                const int kb = kb0 + st * kUG + kbl, R = r0 + row;
                const bool v = R < a.total_rows && kb < kb1;
                const uint8_t *src = a.seg[0].W;
                if (v) {
                    const uint16_t *wsr;
                    int yo;
                    src = urow(a, R, &wsr, &yo) + (size_t)kb * Lay::RB + sub * 16;
                }
                const int slot = pc ^ ((row >> Lay::RSH) & (PPR - 1));
                cp_async16_zfill_l2(base + Lay::raw + buf * Lay::RAWB + row * Lay::RAWS + slot * 16,
                                    src, v);
            }
            for (int i = p; i < Lay::BTB / 16; i += 128) {
                const int kbl = i / (8 * NP), off = i % (8 * NP);
                const int kb = kb0 + st * kUG + kbl;
                const bool v = kb < kb1;
                const uint8_t *src = v ? bprep + (size_t)kb * (128 * NP) + (size_t)off * 16 : bprep;
                cp_async16_zfill(base + Lay::btile + buf * Lay::BTB + i * 16, src, v);
            }
            cp_async_commit();
        };
        for (int st = 0; st < kUPD; st++) issue_stage(st);
        for (int st = 0; st < nst; st++) {
            const int nx = st + kUPD;
            if (p == 0) {
                bool w = true;
                // stage buffer nx % kUStg last held stage nx - kUStg; A buffer
                // st % 2 held stage st - 2: their MMAs must be done
                if (nx < nst && nx >= kUStg)
                    w = umma::mbar_wait(bfree + 8 * (nx % kUStg),
                                        (uint32_t)(nx / kUStg - 1) & 1u, umma::kWaitLimit);
                if (w && st >= 2)
                    w = umma::mbar_wait(afree + 8 * (st & 1), (uint32_t)(st / 2 - 1) & 1u,
                                        umma::kWaitLimit);
                if (!w) {
                    atomicOr(err, 8);
                    s_abort = 1;
                }
                s_stop = s_abort;
            }
            producers_sync();
            if (s_stop) break;
            issue_stage(nx);
            cp_async_wait<kUPD>();                        // this thread's stage st
            producers_sync();                             // everyone's
            {
                const uint8_t *rs = rawb + (st % kUStg) * Lay::RAWB + p * Lay::RAWS;
                const int swz = (p >> Lay::RSH) & (Lay::PPR - 1);
                uint8_t *ad = atb + (st & 1) * Lay::ATB + p * 16;
                constexpr int PB = Lay::RB / 16;                  // pieces per block
#pragma unroll
                for (int kbl = 0; kbl < kUG; kbl++) {
                    const uint4 w0 = *(const uint4 *)(rs + ((kbl * PB) ^ swz) * 16);
                    const uint4 w1 = PB > 1 ? *(const uint4 *)(rs + ((kbl * PB + 1) ^ swz) * 16)
                                            : w0;
                    convert_block<BITS>(w0, w1, ad + kbl * (kURows * 64));
                }
            }
            umma::fence_smem_async();
            producers_sync();
            if (p == 0) mbar_arrive(aready + 8 * (st & 1));
        }
        cp_async_wait<0>();
    } else if (lane == 0) {
        // ---- the MMA warp: per 32-k block, two K = 16 MMAs of N = 2 NP
        // (hi and lo rows of B at once) into the group's accumulator
        const uint32_t idesc = umma::idesc_f16(kURows, 2 * NP);
        const uint64_t ad0 = umma::desc(base + Lay::atile, kURows * 16, 128);
        const uint64_t bd0 = umma::desc(base + Lay::btile, 2 * NP * 16, 128);
        int b = 0, uses = 0;                     // accumulator, and its use count
        int seg_end = (g0 + 1) * gpb < kb1 ? (g0 + 1) * gpb : kb1;
        bool first = true;
        int last = -1;
        bool w = true;
        for (int st = 0; st < nst && w; st++) {
            w = umma::mbar_wait(aready + 8 * (st & 1), (uint32_t)(st / 2) & 1u, umma::kWaitLimit);
            if (!w) break;
            umma::fence_after();
            const uint64_t ad = ad0 + (uint64_t)(((st & 1) * Lay::ATB) >> 4);
            const uint64_t bd = bd0 + (uint64_t)(((st % kUStg) * Lay::BTB) >> 4);
            for (int kbl = 0; kbl < kUG; kbl++) {
                const int kb = kb0 + st * kUG + kbl;
                if (kb >= kb1) break;
                if (first && uses > 0) {
                    w = umma::mbar_wait(empty + 8 * b, (uint32_t)(uses - 1) & 1u, umma::kWaitLimit);
                    if (!w) break;
                    umma::fence_after();
                }
#pragma unroll
                for (int kk = 0; kk < 2; kk++)
                    umma::mma_f16(tmem + (uint32_t)(b * 2 * NP),
                                  ad + (uint64_t)((kbl * (kURows * 64) + kk * (2 * kURows * 16)) >> 4),
                                  bd + (uint64_t)((kbl * (128 * NP) + kk * (2 * 2 * NP * 16)) >> 4),
                                  idesc, !(first && kk == 0));
                first = false;
                if (kb + 1 == seg_end) {
                    umma::commit(full + 8 * b);
                    first = true;
                    seg_end = seg_end + gpb < kb1 ? seg_end + gpb : kb1;
                    if (++b == NBUF) { b = 0; uses++; }
                }
            }
            umma::commit(afree + 8 * (st & 1));
            umma::commit(bfree + 8 * (st % kUStg));
            last = st;
        }
        if (!w) {
            atomicOr(err, 8);
            s_abort = 1;
        }
        if (last >= 0 &&
            !umma::mbar_wait(bfree + 8 * (last % kUStg), (uint32_t)(last / kUStg) & 1u,
                             umma::kWaitLimit))
            atomicOr(err, 8);
    }
    umma::fence_before();
    __syncthreads();
    if (warp == 0) {
        umma::fence_after();
        umma::tmem_free(tmem, Lay::tcols);
    }
}

// Y[t][o] = sum over the S splits, in split order.
__global__ void mvq_umma_reduce_kernel(const MvqArgs a, const float *__restrict__ part, int S) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)a.batch * a.total_rows) return;
    const int t = (int)(i / a.total_rows), R = (int)(i % a.total_rows);
    float v = part[((size_t)0 * a.batch + t) * a.total_rows + R];
    for (int s = 1; s < S; s++) v = __fadd_rn(v, part[((size_t)s * a.batch + t) * a.total_rows + R]);
    const uint16_t *wsr;
    int yo;
    urow(a, R, &wsr, &yo);
    a.Y[(size_t)t * a.y_stride + yo] = v;
}

// ------------------------------------------------------------ host side --

__device__ unsigned g_umma_err;            // bit 2: epilogue wait, bit 3: producer wait

struct UmmaPlan {
    int nkb, NP, S;
    size_t bprep, part;                    // scratch sections, 256-byte multiples
};

static UmmaPlan umma_plan(int batch, int in, int rows) {
    UmmaPlan p;
    p.nkb = (in + 31) / 32;
    p.NP = (batch + 15) / 16 * 16;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int tiles = (rows + kURows - 1) / kURows;
    // the CTAs an SM holds (two up to 32 tokens, else one); at least two
    // stages of work per split
    const int cps = p.NP <= 32 ? 2 : 1;
    int S = (cps * sms) / tiles;
    S = S < 1 ? 1 : S;
    const int smax = p.nkb / (2 * kUG) > 1 ? p.nkb / (2 * kUG) : 1;
    p.S = S < smax ? S : smax;
    p.bprep = ((size_t)p.nkb * 128 * p.NP + 255) / 256 * 256;
    p.part = p.S > 1 ? ((size_t)p.S * batch * rows * 4 + 255) / 256 * 256 : 0;
    return p;
}

size_t mvq_xf_bytes(int batch, int in, int rows) {
    const UmmaPlan p = umma_plan(batch, in, rows);
    return p.bprep + 256 + p.part;
}

template <int BITS, int NPB>
static int launch_umma_np(const MvqArgs &a, const UmmaPlan &p, uint8_t *bprep, float *tscale,
                          float *part, cudaStream_t st) {
    using Lay = ULay<BITS, 16 * NPB>;
    static bool attr_done = false;                   // per instantiation, per process
    auto fn = mvq_umma_kernel<BITS, NPB>;
    if (!attr_done) {
        const cudaError_t e = cudaFuncSetAttribute(
            fn, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::bytes);
        if (e != cudaSuccess) return cuda_fail(e, "mvq umma smem attribute");
        attr_done = true;
    }
    unsigned *err = nullptr;
    cudaError_t e = cudaGetSymbolAddress((void **)&err, g_umma_err);
    if (e != cudaSuccess) return cuda_fail(e, "mvq umma error word");
    const int tiles = (a.total_rows + kURows - 1) / kURows;
    fn<<<tiles * p.S, kUThreads, Lay::bytes, st>>>(a, bprep, tscale, part, p.nkb, p.S, (int *)err);
    WARP_CHECK_LAUNCH("mvq_umma_kernel");
    return WARP_OK;
}

int launch_umma(const MvqArgs &a, cudaStream_t st) {
    const UmmaPlan p = umma_plan(a.batch, a.in, a.total_rows);
    uint8_t *bprep = (uint8_t *)a.xf;
    float *tscale = (float *)(bprep + p.bprep);
    float *part = (float *)(bprep + p.bprep + 256);
    // about four CTAs per SM over (token row, share of the k-groups)
    int shares = (4 * 148) / p.NP;
    shares = shares < 1 ? 1 : shares > p.nkb ? p.nkb : shares;
    mvq_umma_prep_kernel<<<dim3(p.NP, shares), 256, 0, st>>>(a, bprep, tscale, p.nkb, p.NP);
    WARP_CHECK_LAUNCH("mvq_umma_prep_kernel");
    int rc;
    const int npb = p.NP / 16;
    if (a.bits == 4)
        rc = npb == 1 ? launch_umma_np<4, 1>(a, p, bprep, tscale, part, st)
           : npb == 2 ? launch_umma_np<4, 2>(a, p, bprep, tscale, part, st)
           : npb == 3 ? launch_umma_np<4, 3>(a, p, bprep, tscale, part, st)
                      : launch_umma_np<4, 4>(a, p, bprep, tscale, part, st);
    else
        rc = npb == 1 ? launch_umma_np<8, 1>(a, p, bprep, tscale, part, st)
           : npb == 2 ? launch_umma_np<8, 2>(a, p, bprep, tscale, part, st)
           : npb == 3 ? launch_umma_np<8, 3>(a, p, bprep, tscale, part, st)
                      : launch_umma_np<8, 4>(a, p, bprep, tscale, part, st);
    if (rc || p.S == 1) return rc;
    const size_t n = (size_t)a.batch * a.total_rows;
    mvq_umma_reduce_kernel<<<cdiv(n, 256), 256, 0, st>>>(a, part, p.S);
    WARP_CHECK_LAUNCH("mvq_umma_reduce_kernel");
    return WARP_OK;
}

}  // namespace warp

extern "C" int warp_mvq_status(int clear) {
    unsigned v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, warp::g_umma_err, sizeof(v));
    if (e != cudaSuccess) return warp::cuda_fail(e, "warp_mvq_status");
    if (clear && v) {
        const unsigned z = 0;
        e = cudaMemcpyToSymbol(warp::g_umma_err, &z, sizeof(z));
        if (e != cudaSuccess) return warp::cuda_fail(e, "warp_mvq_status");
    }
    if (v) {
        warp::set_error("mvq: a tensor-core matmul wait gave up (flags 0x%x)", v);
        return WARP_E_TIMEOUT;
    }
    return WARP_OK;
}
