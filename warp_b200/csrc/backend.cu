// backend.cu — the reference engine's plugin boundary, host pointers in.
//
//  * waste_register_cuda: fills the engine's waste_kernels table
//    (waste_backend.h:69-107) the way backend.c:169-219 expects of an
//    accelerator: it is called after the SIMD kernels registered and after
//    mvq_rows_cpu was snapshotted (backend.c:202, 209), overwrites only the
//    slot it implements (mvq_rows_f32), sets on_device so run_rows
//    (model.c:805-813) hands it whole matrices from one thread, and returns a
//    name, or NULL to decline.
//  * waste_cuda_vq3r: the batch VQ3R apply with the job ABI of
//    waste_metal_vq3r (waste_metal.h:25-44); never partially applied.
//  * waste_cuda_release_host_buffers: drops the device mirrors
//    (backend.c:229-235).
//
// Weights arrive as host pointers owned by the engine and do not change for
// the life of a model, so each trunk tensor is mirrored to the device once,
// keyed by its host address and size.  Expert records live in cache slots
// that are reused for other experts, so they are keyed by what the record
// says it is (layer, expert id, codebook, checksum), never by address.
#include "common.cuh"
#include "mvq.cuh"
#include "vq_gather.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

namespace warp {

// waste_kernels (waste_backend.h:69-107), field for field: the engine hands
// us a pointer to its table and this is the layout it has.
struct EngineKernels {
    void (*kda_step)(int, int, int, const float *, const float *, const float *,
                     const float *, const float *, float *, float *, float *);
    void (*short_conv_step)(int, int, const float *, const float *, float *,
                            const float *, float *);
    void (*rmsnorm_gated)(int, const float *, const float *, const float *, float,
                          float *);
    void (*mvq_rows_f32)(int, int, void *);
    void (*lutb_range)(int, int, void *);
    void (*vq_rows_p6)(int, int, void *);
    void (*vq_rows_e)(int, int, void *);
    int on_device;
    void (*mvq_rows_cpu)(int, int, void *);
    size_t device_min_bytes;
};

// mvq_arg (simd.h:35-39).
struct EngineMvqArg {
    float *y;
    const int8_t *W;
    const uint16_t *ws;
    const int8_t *xq;
    const float *xs;
    int in, ng, group, bits;
    size_t rowbytes;
};

struct Mirror {
    void *dev;
    size_t bytes;
};

static std::mutex g_mu;
static std::map<std::pair<const void *, size_t>, Mirror> g_trunk;
static std::map<std::tuple<uint32_t, uint32_t, uint32_t, size_t>, Mirror> g_recs;
static void (*g_cpu_mvq)(int, int, void *) = nullptr;
static int g_dev = -1;
static cudaStream_t g_stream = nullptr;
static void *g_scratch = nullptr;
static size_t g_scratch_cap = 0;
static unsigned long long g_fallbacks = 0;
static unsigned long long g_mvq_device = 0;      // slot calls the device ran
static unsigned long long g_vq3r_calls = 0, g_vq3r_jobs = 0;

static void *scratch(size_t bytes) {
    if (bytes <= g_scratch_cap) return g_scratch;
    if (g_scratch) cudaFree(g_scratch);
    g_scratch = nullptr;
    g_scratch_cap = 0;
    size_t cap = bytes < ((size_t)1 << 20) ? ((size_t)1 << 20) : bytes;
    if (cudaMalloc(&g_scratch, cap) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    g_scratch_cap = cap;
    return g_scratch;
}

static void *mirror_trunk(const void *host, size_t bytes) {
    auto key = std::make_pair(host, bytes);
    auto it = g_trunk.find(key);
    if (it != g_trunk.end()) return it->second.dev;
    void *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) { cudaGetLastError(); return nullptr; }
    if (cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(d);
        return nullptr;
    }
    g_trunk[key] = {d, bytes};
    return d;
}

// The device matvec behind waste_k.mvq_rows_f32.  Rows [b, e) of the
// matrix; any shape the kernel does not take (3-bit rows, a row stride that
// is not a whole number of 16-byte chunks) and any device failure run the
// engine's own CPU kernel instead, which is the table's contract: every slot
// must produce a result (waste_backend.h:23-27; metal.m:285-304 does the
// same).  warp_cuda_fallback_count() reports how often that happened.
static void mvq_rows_cuda(int b, int e, void *p) {
    EngineMvqArg *a = (EngineMvqArg *)p;
    if (e <= b) return;
    const int rows = e - b;
    bool ok = (a->bits == 4 || a->bits == 8) && a->rowbytes % 16 == 0 &&
              a->group % 32 == 0 && a->in > 0;
    if (ok) {
        std::lock_guard<std::mutex> lk(g_mu);
        cudaSetDevice(g_dev);
        const size_t wbytes = (size_t)e * a->rowbytes;
        const size_t sbytes = (size_t)e * a->ng * sizeof(uint16_t);
        const uint8_t *dW = (const uint8_t *)mirror_trunk(a->W, wbytes);
        const uint16_t *dS = (const uint16_t *)mirror_trunk(a->ws, sbytes);
        const size_t xb = ((size_t)a->in * 4 + 255) & ~(size_t)255;
        const size_t yb = ((size_t)rows * 4 + 255) & ~(size_t)255;
        uint8_t *s = (uint8_t *)scratch(xb + yb);
        ok = dW && dS && s;
        if (ok) {
            float *dx = (float *)s, *dy = (float *)(s + xb);
            MvqArgs m = {};
            m.seg[0] = {dW + (size_t)b * a->rowbytes, dS + (size_t)b * a->ng, rows, 0};
            m.nseg = 1;
            m.in = a->in;
            m.group = a->group;
            m.bits = a->bits;
            m.rowbytes = a->rowbytes;
            m.batch = 1;
            m.X = dx;
            m.Y = dy;
            m.y_stride = rows;
            ok = cudaMemcpyAsync(dx, a->xs, (size_t)a->in * 4, cudaMemcpyHostToDevice,
                                 g_stream) == cudaSuccess &&
                 mvq_launch(m, g_stream) == WARP_OK &&
                 cudaMemcpyAsync(a->y + b, dy, (size_t)rows * 4, cudaMemcpyDeviceToHost,
                                 g_stream) == cudaSuccess &&
                 cudaStreamSynchronize(g_stream) == cudaSuccess;
            if (!ok) cudaGetLastError();
            else g_mvq_device++;
        }
    }
    if (!ok) {
        {
            std::lock_guard<std::mutex> lk(g_mu);
            g_fallbacks++;
        }
        if (g_cpu_mvq) g_cpu_mvq(b, e, p);
    }
}

}  // namespace warp

using namespace warp;

// WARP_CUDA_STATS=<path>: at exit, one JSON line of the boundary's counters
// is appended to <path> (for a harness that runs the engine in its own
// process and wants to know the device did the work).
static void stats_at_exit() {
    const char *path = getenv("WARP_CUDA_STATS");
    if (!path || !*path) return;
    FILE *f = fopen(path, "a");
    if (!f) return;
    fprintf(f,
            "{\"mvq_device\": %llu, \"mvq_fallback\": %llu, \"vq3r_calls\": %llu, "
            "\"vq3r_jobs\": %llu}\n",
            g_mvq_device, g_fallbacks, g_vq3r_calls, g_vq3r_jobs);
    fclose(f);
}

extern "C" const char *waste_register_cuda(void *table) {
    if (!table) return nullptr;
    const char *off = getenv("WARP_CUDA_DISABLE");
    if (off && *off && *off != '0') return nullptr;
    int dev = 0;
    if (const char *s = getenv("WARP_CUDA_DEVICE")) dev = atoi(s);
    if (!warp_device_ok(dev)) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    EngineKernels *t = (EngineKernels *)table;
    if (g_dev < 0) {
        if (cudaSetDevice(dev) != cudaSuccess ||
            cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_dev = dev;
        if (getenv("WARP_CUDA_STATS")) atexit(stats_at_exit);
    }
    // Idempotent: a second registration must not snapshot our own slot as
    // the CPU kernel.
    if (t->mvq_rows_f32 != mvq_rows_cuda) g_cpu_mvq = t->mvq_rows_cpu ? t->mvq_rows_cpu
                                                                      : t->mvq_rows_f32;
    t->mvq_rows_f32 = mvq_rows_cuda;
    t->on_device = 1;
    // Below this many weight bytes the pool's CPU kernel is faster than a
    // device round trip (the engine's own device_min_bytes rule,
    // waste_backend.h:102-104).  WARP_CUDA_DEVICE_MIN_KB overrides.
    long kb = 256;
    if (const char *s = getenv("WARP_CUDA_DEVICE_MIN_KB")) kb = atol(s);
    t->device_min_bytes = kb < 0 ? (size_t)-1 : (size_t)kb << 10;
    return "CUDA sm_100a";
}

extern "C" unsigned long long warp_cuda_fallback_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_fallbacks;
}

extern "C" void waste_cuda_release_host_buffers(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_dev >= 0) cudaSetDevice(g_dev);
    for (auto &kv : g_trunk) cudaFree(kv.second.dev);
    g_trunk.clear();
    for (auto &kv : g_recs) cudaFree(kv.second.dev);
    g_recs.clear();
    if (g_scratch) cudaFree(g_scratch);
    g_scratch = nullptr;
    g_scratch_cap = 0;
}


// waste_metal_vq3r's contract on CUDA: every job's y = scale * sum_v
// (T0 + T1) + T2 in the CPU's order (bit-identical to vq_rows, as the Metal
// kernel is, metal.m:130-137), all outputs staged on the device and copied
// back only when every job ran.
extern "C" int waste_cuda_vq3r(const warp_vq_job *jobs, int n) {
    if (!jobs || n <= 0 || g_dev < 0) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaSetDevice(g_dev);
    size_t ytotal = 0;
    std::map<const float *, std::pair<size_t, size_t>> luts;   // host -> (bytes, offset)
    size_t lut_total = 0;
    for (int i = 0; i < n; i++) {
        const warp_vq_job &j = jobs[i];
        if (j.stages != 3 || j.entries != 256 || j.m <= 0 || j.nv <= 0 || !j.rec ||
            !j.lut || j.rec_bytes < 48 || !j.y)
            return -1;
        // every byte a job reads lies inside the buffers it names: the
        // blocked indices and the fp16 scales in the record, nv tables of
        // 3 x 256 floats from lut_off in the LUT
        const size_t idx_bytes = (size_t)((j.m + 63) / 64) * (size_t)j.nv * 64 * 3;
        if ((size_t)j.idx_off + idx_bytes > j.rec_bytes || j.sc_off % 2 != 0 ||
            (size_t)j.sc_off + 2 * (size_t)j.m > j.rec_bytes ||
            ((size_t)j.lut_off + (size_t)j.nv * 3 * 256) * sizeof(float) > j.lut_bytes)
            return -1;
        ytotal += (size_t)j.m;
        if (!luts.count(j.lut)) {
            luts[j.lut] = {j.lut_bytes, lut_total};
            lut_total += (j.lut_bytes + 255) & ~(size_t)255;
        }
    }
    uint8_t *s = (uint8_t *)scratch(lut_total + ytotal * 4 + 256);
    if (!s) return -1;
    for (auto &kv : luts)
        if (cudaMemcpyAsync(s + kv.second.second, kv.first, kv.second.first,
                            cudaMemcpyHostToDevice, g_stream) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
    float *dy = (float *)(s + lut_total);
    size_t yoff = 0;
    for (int i = 0; i < n; i++) {
        const warp_vq_job &j = jobs[i];
        uint32_t hdr[12];
        memcpy(hdr, j.rec, sizeof hdr);
        // (layer | expert_id), codebook_id, crc32, size
        auto key = std::make_tuple(hdr[1], hdr[2] >> 16, hdr[9], j.rec_bytes);
        void *drec = nullptr;
        auto it = g_recs.find(key);
        if (it != g_recs.end()) drec = it->second.dev;
        else {
            if (cudaMalloc(&drec, j.rec_bytes) != cudaSuccess ||
                cudaMemcpy(drec, j.rec, j.rec_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
                cudaGetLastError();
                if (drec) cudaFree(drec);
                return -1;
            }
            g_recs[key] = {drec, j.rec_bytes};
        }
        const float *dl = (const float *)(s + luts[j.lut].second) + j.lut_off;
        if (vq_apply_ordered_launch(dy + yoff, (const uint8_t *)drec + j.idx_off,
                                    (const uint16_t *)((const uint8_t *)drec + j.sc_off),
                                    dl, j.m, j.nv, g_stream) != WARP_OK)
            return -1;
        yoff += (size_t)j.m;
    }
    std::vector<float> hy(ytotal);
    if (cudaMemcpyAsync(hy.data(), dy, ytotal * 4, cudaMemcpyDeviceToHost, g_stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(g_stream) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    yoff = 0;
    for (int i = 0; i < n; i++) {
        memcpy(jobs[i].y, hy.data() + yoff, (size_t)jobs[i].m * 4);
        yoff += (size_t)jobs[i].m;
    }
    g_vq3r_calls++;
    g_vq3r_jobs += (unsigned long long)n;
    return 0;
}

// ---- the engine's Metal hooks, answered by CUDA ----------------------------
//
// model.c reaches the routed-expert apply only through the Metal batch hook
// (model.c:5665-5792, under WASTE_ENABLE_METAL and WASTE_METAL_MOE=1), and
// backend.c registers Metal and releases its mirrors under the same flag
// (backend.c:54-56, 211-213, 229-235).  Exporting these three symbols lets
// the reference build with -DWASTE_ENABLE_CUDA=1 -DWASTE_ENABLE_METAL=1 and
// link this library in place of src/metal.m, with model.c and backend.c
// unchanged: registration then goes to CUDA (waste_register_cuda runs
// first), the Metal registration declines, and the batch hook runs here.

extern "C" int waste_metal_vq3r(const warp_vq_job *jobs, int n) {
    return waste_cuda_vq3r(jobs, n);
}

extern "C" const char *waste_register_metal(void *table) {
    (void)table;
    return nullptr;                 // no Metal device; CUDA registered already
}

extern "C" void waste_metal_release_host_buffers(void) {
    waste_cuda_release_host_buffers();
}

// waste_metal_selftest (metal.m:403-460): a dispatch-rate diagnostic the
// engine runs only when WASTE_METAL_SELFTEST is set (test_forward.c:271-275).
// Its contract is to measure the trunk Q4 matvec the backend runs (M 12288,
// K 7168, group 128) and print the rates to stderr; this is the CUDA
// version: device-resident weights reused, the same rotated over 32 copies
// (so every launch reads HBM), and rotated with the x / y host copies of a
// slot call included.  Nothing is returned and nothing else is touched.
extern "C" void waste_metal_selftest(void) {
    if (g_dev < 0) return;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaSetDevice(g_dev);
    const int M = 12288, K = 7168, G = 128, ng = K / G, NC = 32, R = 64;
    const size_t rb = K / 2, wb = (size_t)M * rb, sb = (size_t)M * ng * 2;
    std::vector<void *> w(NC, nullptr), sc(NC, nullptr);
    float *x = nullptr, *y = nullptr;
    std::vector<float> hx(K, 0.01f), hy(M);
    bool ok = cudaMalloc((void **)&x, K * 4) == cudaSuccess &&
              cudaMalloc((void **)&y, M * 4) == cudaSuccess;
    for (int i = 0; ok && i < NC; i++)
        ok = cudaMalloc(&w[i], wb) == cudaSuccess && cudaMalloc(&sc[i], sb) == cudaSuccess &&
             cudaMemset(w[i], 0x37 + i, wb) == cudaSuccess &&
             cudaMemset(sc[i], 0x38, sb) == cudaSuccess;
    ok = ok && cudaMemcpy(x, hx.data(), K * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    ok = ok && cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
    const char *nm[3] = {"device buf, reused ", "device buf, 32 rot ", "32 rot + x/y memcpy"};
    for (int mode = 0; ok && mode < 3; mode++) {
        double best = 1e18, sum = 0;
        for (int r = 0; ok && r < R; r++) {
            const int c = mode == 0 ? 0 : r % NC;
            MvqArgs m = {};
            m.seg[0] = {(const uint8_t *)w[c], (const uint16_t *)sc[c], M, 0};
            m.nseg = 1;
            m.in = K;
            m.group = G;
            m.bits = 4;
            m.rowbytes = rb;
            m.batch = 1;
            m.X = x;
            m.Y = y;
            m.y_stride = M;
            ok = cudaEventRecord(e0, g_stream) == cudaSuccess;
            if (mode == 2)
                ok = ok && cudaMemcpyAsync(x, hx.data(), K * 4, cudaMemcpyHostToDevice,
                                           g_stream) == cudaSuccess;
            ok = ok && mvq_launch(m, g_stream) == WARP_OK;
            if (mode == 2)
                ok = ok && cudaMemcpyAsync(hy.data(), y, M * 4, cudaMemcpyDeviceToHost,
                                           g_stream) == cudaSuccess;
            ok = ok && cudaEventRecord(e1, g_stream) == cudaSuccess &&
                 cudaEventSynchronize(e1) == cudaSuccess;
            float ms = 0.0f;
            ok = ok && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess;
            const double dt = ms * 1e-3;
            if (dt < best) best = dt;
            if (r >= 8) sum += dt;
        }
        if (ok)
            fprintf(stderr, "warp_b200: cuda selftest %s  mean %.3f ms %6.1f GB/s  best %6.1f GB/s\n",
                    nm[mode], sum / (R - 8) * 1e3, wb / (sum / (R - 8)) / 1e9, wb / best / 1e9);
    }
    if (!ok) cudaGetLastError();
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    for (int i = 0; i < NC; i++) {
        if (w[i]) cudaFree(w[i]);
        if (sc[i]) cudaFree(sc[i]);
    }
    if (x) cudaFree(x);
    if (y) cudaFree(y);
}

extern "C" int warp_cuda_stats(unsigned long long *out) {
    if (!out) return WARP_E_ARG;
    std::lock_guard<std::mutex> lk(g_mu);
    out[0] = g_mvq_device;
    out[1] = g_fallbacks;
    out[2] = g_vq3r_calls;
    out[3] = g_vq3r_jobs;
    return WARP_OK;
}
