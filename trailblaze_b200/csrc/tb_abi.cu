// tb_abi.cu — the exported C ABI (include/tb_gguf_dequant.h).
//
// Part 1 keeps the reference's layer4/tb_gguf_dequant.h:19-43 contract.  What
// differs from layer4/tb_gguf_dequant.cu:337-486 is inside: one non-blocking
// library stream instead of four round-robin streams whose pipelining the
// per-call synchronize defeated (.cu:437-467); pinned host staging for x and y
// so the two copies per call are DMA transfers; a device-resident x that
// tb_cuda_upload_x really fills and tb_cuda_matvec_device(x_host = NULL) really
// reads; launch geometry that never depends on the oscillator snapshot; and a
// mutex, so concurrent callers are serialised instead of racing on static
// buffers.  Errors return 0 / NULL with a message on stderr; nothing aborts.
//
// Host-side fault injection for tests: TB_CUDA_FAULT=alloc|copy|launch makes
// tb_cuda_upload_tensor, the H2D copy of tb_cuda_matvec_device, or its kernel
// launch fail (return 0/NULL) without touching the GPU.  TB_WAIT_LIMIT sets
// the poll limit of the kernels' bounded pipeline waits.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "../../include/tb_gguf_dequant.h"
#include "tb_common.cuh"
#include "tb_internal.h"

namespace {

struct State {
    int dev = -1;
    int num_sms = 0;
    cudaStream_t stream = nullptr;
    int *d_err = nullptr;       // device error word
    int *h_err = nullptr;       // pinned copy of it
    float *d_x = nullptr, *d_y = nullptr;
    float *h_x = nullptr, *h_y = nullptr;   // pinned staging
    size_t cap_x = 0, cap_y = 0;            // element capacity of the four buffers above
    int x_loaded = 0;                        // K of the vector tb_cuda_upload_x left in d_x
    uint32_t wait_limit = 1u << 22;
    int fault = 0;                           // 1 alloc, 2 copy, 3 launch
    tb::SmpScratch smp;                      // two-stage top-k candidates (first sampling call)
};

State g;
std::mutex g_mu;
std::atomic<unsigned long long> g_launches{0};

bool cuda_ok(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return true;
    fprintf(stderr, "[tb_cuda] %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

void read_env()
{
    const char *f = getenv("TB_CUDA_FAULT");
    g.fault = !f ? 0 : !strcmp(f, "alloc") ? 1 : !strcmp(f, "copy") ? 2 : !strcmp(f, "launch") ? 3 : 0;
    const char *w = getenv("TB_WAIT_LIMIT");
    if (w && atol(w) > 0) g.wait_limit = static_cast<uint32_t>(atol(w));
}

// Binds the current device and creates the stream and error word.  Caller holds g_mu.
bool ensure_init_locked(bool verbose)
{
    int cur = 0;
    if (!cuda_ok(cudaGetDevice(&cur), "cudaGetDevice")) return false;
    if (g.dev == cur && g.stream) return true;
    if (g.stream) return g.dev == cur;   // initialised on another device: keep the first binding
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return false;
    if (!cuda_ok(cudaSetDevice(cur), "cudaSetDevice")) return false;
    read_env();
    if (!cuda_ok(cudaDeviceGetAttribute(&g.num_sms, cudaDevAttrMultiProcessorCount, cur), "sm count"))
        return false;
    if (!cuda_ok(cudaStreamCreateWithFlags(&g.stream, cudaStreamNonBlocking), "stream")) return false;
    if (!cuda_ok(cudaMalloc(&g.d_err, sizeof(int)), "err alloc")) return false;
    if (!cuda_ok(cudaMallocHost(&g.h_err, sizeof(int)), "err pin")) return false;
    cudaMemset(g.d_err, 0, sizeof(int));
    *g.h_err = 0;
    g.dev = cur;
    if (verbose) {
        cudaDeviceProp p;
        cudaGetDeviceProperties(&p, cur);
        size_t fm = 0, tm = 0;
        cudaMemGetInfo(&fm, &tm);
        printf("[tb_cuda] %s sm_%d%d  %d SMs  %.1f GB total  %.1f GB free  (%s)\n", p.name, p.major,
               p.minor, g.num_sms, tm / 1e9, fm / 1e9, tb_cuda_version());
    }
    return true;
}

bool grow(size_t K, size_t M)
{
    if (K > g.cap_x) {
        if (g.d_x) cudaFree(g.d_x);
        if (g.h_x) cudaFreeHost(g.h_x);
        g.d_x = nullptr; g.h_x = nullptr; g.cap_x = 0; g.x_loaded = 0;
        if (!cuda_ok(cudaMalloc(&g.d_x, K * sizeof(float)), "x alloc")) return false;
        if (!cuda_ok(cudaMallocHost(&g.h_x, K * sizeof(float)), "x pin")) return false;
        g.cap_x = K;
    }
    if (M > g.cap_y) {
        if (g.d_y) cudaFree(g.d_y);
        if (g.h_y) cudaFreeHost(g.h_y);
        g.d_y = nullptr; g.h_y = nullptr; g.cap_y = 0;
        if (!cuda_ok(cudaMalloc(&g.d_y, M * sizeof(float)), "y alloc")) return false;
        if (!cuda_ok(cudaMallocHost(&g.h_y, M * sizeof(float)), "y pin")) return false;
        g.cap_y = M;
    }
    return true;
}

// ---- static device staging of tb_cuda_matvec_device_noalloc ----
// One fixed set per device, fixed at build time: x up to kNaMaxK floats
// (256 KB), y up to kNaMaxM floats (1 MB), and the device error word.
constexpr int kNaMaxK = 65536;
constexpr int kNaMaxM = 262144;
__device__ __align__(256) float g_na_x[kNaMaxK];
__device__ __align__(256) float g_na_y[kNaMaxM];
__device__ __align__(256) int g_na_err[64];

struct NaDev {
    int dev;
    int sms;
    float *x, *y;
    int *err;
};
NaDev g_na[32];
int g_nna = 0;

// Addresses of the static buffers on the current device, looked up once per
// device (cudaGetSymbolAddress; nothing is allocated).  Caller holds g_mu.
const NaDev *na_device_locked()
{
    int dev = 0;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return nullptr;
    for (int i = 0; i < g_nna; ++i)
        if (g_na[i].dev == dev) return &g_na[i];
    if (g_nna == 32) return nullptr;
    NaDev d{};
    d.dev = dev;
    void *px = nullptr, *py = nullptr, *pe = nullptr;
    if (!cuda_ok(cudaGetSymbolAddress(&px, g_na_x), "symbol x") ||
        !cuda_ok(cudaGetSymbolAddress(&py, g_na_y), "symbol y") ||
        !cuda_ok(cudaGetSymbolAddress(&pe, g_na_err), "symbol err") ||
        !cuda_ok(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev), "sm count"))
        return nullptr;
    d.x = static_cast<float *>(px);
    d.y = static_cast<float *>(py);
    d.err = static_cast<int *>(pe);
    g_na[g_nna] = d;
    return &g_na[g_nna++];
}

}  // namespace

namespace tb {
bool smem_attr_once(const void *kernel, int bytes)
{
    // remembers (kernel, device) pairs so the attribute is set once per device
    int dev = 0;
    cudaGetDevice(&dev);
    static std::mutex mu;
    static const void *seen[256];
    static int seen_dev[256];
    static int nseen = 0;
    std::lock_guard<std::mutex> lk(mu);
    for (int i = 0; i < nseen; ++i)
        if (seen[i] == kernel && seen_dev[i] == dev) return true;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return false;
    if (nseen < 256) {
        seen[nseen] = kernel;
        seen_dev[nseen] = dev;
        ++nseen;
    }
    return true;
}
}  // namespace tb

extern "C" {

const char *tb_cuda_version(void) { return "tb_cuda_sm100 1.1 sm_100a"; }

int tb_cuda_qtype_info(int qtype, int *block_weights, int *block_bytes)
{
    const tb::Geom gg = tb::geom_of(qtype);
    if (!gg.block_weights) return 0;
    if (block_weights) *block_weights = gg.block_weights;
    if (block_bytes) *block_bytes = gg.block_bytes;
    return 1;
}

int tb_cuda_init(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (g.stream) return 1;
    return ensure_init_locked(true) ? 1 : 0;
}

void *tb_cuda_upload_tensor(const void *host_data, size_t byte_count)
{
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return nullptr;
        if (g.fault == 1) {
            fprintf(stderr, "[tb_cuda] upload_tensor: injected allocation fault\n");
            return nullptr;
        }
    }
    if (!host_data || byte_count == 0) return nullptr;
    void *d = nullptr;
    if (!cuda_ok(cudaMalloc(&d, byte_count), "upload_tensor alloc")) return nullptr;
    if (!cuda_ok(cudaMemcpy(d, host_data, byte_count, cudaMemcpyHostToDevice), "upload_tensor copy")) {
        cudaFree(d);
        return nullptr;
    }
    return d;
}

void tb_cuda_free_tensor(void *d_ptr)
{
    if (d_ptr) cudaFree(d_ptr);
}

int tb_cuda_upload_x(const float *x_host, int K)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!x_host || K <= 0 || !ensure_init_locked(false)) return 0;
    if (!grow(static_cast<size_t>(K), 1)) return 0;
    memcpy(g.h_x, x_host, static_cast<size_t>(K) * sizeof(float));
    if (!cuda_ok(cudaMemcpyAsync(g.d_x, g.h_x, static_cast<size_t>(K) * sizeof(float),
                                 cudaMemcpyHostToDevice, g.stream), "upload_x"))
        return 0;
    if (!cuda_ok(cudaStreamSynchronize(g.stream), "upload_x sync")) return 0;
    g.x_loaded = K;
    return 1;
}

void tb_cuda_set_snap(const void *snap) { (void)snap; }

int tb_cuda_matvec_device(const void *W_device, int qtype, int M, int K, const float *x_host,
                          float *out_host)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!W_device || !out_host || M <= 0 || K <= 0) return 0;
    const tb::Geom gg = tb::geom_of(qtype);
    if (!gg.block_weights || K % gg.block_weights) return 0;
    if (!ensure_init_locked(false)) return 0;
    if (!grow(static_cast<size_t>(K), static_cast<size_t>(M))) return 0;
    const size_t xb = static_cast<size_t>(K) * sizeof(float), yb = static_cast<size_t>(M) * sizeof(float);
    if (x_host) {
        if (g.fault == 2) {
            fprintf(stderr, "[tb_cuda] matvec_device: injected copy fault\n");
            return 0;
        }
        memcpy(g.h_x, x_host, xb);
        if (!cuda_ok(cudaMemcpyAsync(g.d_x, g.h_x, xb, cudaMemcpyHostToDevice, g.stream), "x H2D"))
            return 0;
        g.x_loaded = 0;
    } else if (g.x_loaded != K) {
        fprintf(stderr, "[tb_cuda] matvec_device: x_host NULL but no uploaded x of length %d\n", K);
        return 0;
    }
    if (g.fault == 3) {
        fprintf(stderr, "[tb_cuda] matvec_device: injected launch fault\n");
        return 0;
    }
    if (!tb::mv_launch(W_device, qtype, M, K, g.d_x, g.d_y, g.stream, g.d_err, g.num_sms, g.wait_limit))
        return 0;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (!cuda_ok(cudaMemcpyAsync(g.h_y, g.d_y, yb, cudaMemcpyDeviceToHost, g.stream), "y D2H")) return 0;
    if (!cuda_ok(cudaMemcpyAsync(g.h_err, g.d_err, sizeof(int), cudaMemcpyDeviceToHost, g.stream), "err D2H"))
        return 0;
    if (!cuda_ok(cudaStreamSynchronize(g.stream), "matvec sync")) return 0;
    if (*g.h_err != 0) {
        // reported here through the 0 return; cleared so the next call starts clean
        fprintf(stderr, "[tb_cuda] matvec_device: device error %d\n", *g.h_err);
        *g.h_err = 0;
        cudaMemsetAsync(g.d_err, 0, sizeof(int), g.stream);
        cudaStreamSynchronize(g.stream);
        return 0;
    }
    memcpy(out_host, g.h_y, yb);
    return 1;
}

void tb_cuda_sync_all(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (g.stream) cudaStreamSynchronize(g.stream);
}

void tb_cuda_cleanup(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (g.stream) {
        cudaStreamSynchronize(g.stream);
        cudaStreamDestroy(g.stream);
    }
    if (g.d_x) cudaFree(g.d_x);
    if (g.d_y) cudaFree(g.d_y);
    if (g.h_x) cudaFreeHost(g.h_x);
    if (g.h_y) cudaFreeHost(g.h_y);
    if (g.d_err) cudaFree(g.d_err);
    if (g.h_err) cudaFreeHost(g.h_err);
    if (g.smp.cv) cudaFree(g.smp.cv);
    if (g.smp.ci) cudaFree(g.smp.ci);
    if (g.smp.nonfin) cudaFree(g.smp.nonfin);
    g = State{};
}

int tb_cuda_matvec_dev(const void *W_dev, int qtype, int M, int K, const float *d_x, float *d_y,
                       void *stream)
{
    int nsm;
    int *derr;
    uint32_t lim;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return 0;
        nsm = g.num_sms;
        derr = g.d_err;
        lim = g.wait_limit;
    }
    const int r = tb::mv_launch(W_dev, qtype, M, K, d_x, d_y, static_cast<cudaStream_t>(stream), derr,
                                nsm, lim);
    if (r) g_launches.fetch_add(1, std::memory_order_relaxed);
    return r;
}

int tb_cuda_qgemm_dev(const void *W_dev, int qtype, int N, int K, const void *A_bf16_dev, int T, float *C_dev,
                      void *stream)
{
    int nsm;
    int *derr;
    uint32_t lim;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return 0;
        nsm = g.num_sms;
        derr = g.d_err;
        lim = g.wait_limit;
    }
    const int r = tb::qg_launch(W_dev, qtype, N, K, A_bf16_dev, T, C_dev, static_cast<cudaStream_t>(stream), derr,
                                nsm, lim);
    if (r) g_launches.fetch_add(1, std::memory_order_relaxed);
    return r;
}

int tb_cuda_matvec_experts_dev(const void *W_dev, int qtype, int M, int K, int n_experts, const int *d_ids,
                               int n_sel, const float *d_x, int x_stride, float *d_y, int y_stride, int ymode,
                               void *stream)
{
    int nsm;
    int *derr;
    uint32_t lim;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return 0;
        nsm = g.num_sms;
        derr = g.d_err;
        lim = g.wait_limit;
    }
    const tb::Geom gm = tb::geom_of(qtype);
    if (!gm.block_weights || M <= 0 || K <= 0 || K % gm.block_weights || n_experts < 1 || n_sel < 1 ||
        x_stride < 0 || y_stride < 0 || ymode < 0 || ymode > 1)
        return 0;
    const int out = ymode == 1 ? M / 2 : M;
    if ((n_sel > 1 && y_stride < out) || (!d_ids && n_sel > n_experts)) return 0;
    tb::MvFuse f;
    f.ymode = static_cast<uint32_t>(ymode);
    f.ng = static_cast<uint32_t>(n_sel);
    f.n_experts = static_cast<uint32_t>(n_experts);
    f.ids = d_ids;
    f.w_stride = static_cast<unsigned long long>(M) * (K / gm.block_weights) * gm.block_bytes;
    f.x_stride = static_cast<uint32_t>(x_stride);
    f.y_stride = static_cast<uint32_t>(y_stride);
    const int r = tb::mv_launch(W_dev, qtype, M, K, d_x, d_y, static_cast<cudaStream_t>(stream), derr, nsm, lim, &f);
    if (r) g_launches.fetch_add(1, std::memory_order_relaxed);
    return r;
}

int tb_cuda_sample_dev(const float *d_logits, int vocab, int top_k, float top_p, float temperature, float u,
                       int *d_token, void *stream)
{
    int *derr;
    tb::SmpScratch scr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return 0;
        derr = g.d_err;
        if (!g.smp.cv && top_k > 0) {   // the two-stage top-k's candidates; without them one CTA does it
            if (cudaMalloc(&g.smp.cv, sizeof(float) * tb::kSmpPreCap) != cudaSuccess ||
                cudaMalloc(&g.smp.ci, sizeof(int) * tb::kSmpPreCap) != cudaSuccess ||
                cudaMalloc(&g.smp.nonfin, sizeof(int)) != cudaSuccess ||
                cudaMemset(g.smp.nonfin, 0, sizeof(int)) != cudaSuccess) {
                cudaGetLastError();
                if (g.smp.cv) cudaFree(g.smp.cv);
                if (g.smp.ci) cudaFree(g.smp.ci);
                if (g.smp.nonfin) cudaFree(g.smp.nonfin);
                g.smp = tb::SmpScratch{};
            }
        }
        scr = g.smp;
    }
    const int r = tb::sample_launch(d_logits, vocab, top_k, top_p, temperature, u, d_token, derr,
                                    static_cast<cudaStream_t>(stream), nullptr, nullptr, nullptr, nullptr, &scr);
    if (r) g_launches.fetch_add(1, std::memory_order_relaxed);
    return r;
}

int tb_cuda_matvec_fused_dev(const void *W_dev, int qtype, int M, int K, const float *d_x, float *d_y,
                             int xmode, const float *d_x2, const float *d_norm_w, float eps,
                             const float *d_res, int ymode, void *stream)
{
    int nsm;
    int *derr;
    uint32_t lim;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return 0;
        nsm = g.num_sms;
        derr = g.d_err;
        lim = g.wait_limit;
    }
    if (xmode < 0 || ymode < 0) return 0;
    tb::MvFuse f;
    f.xmode = static_cast<uint32_t>(xmode);
    f.ymode = static_cast<uint32_t>(ymode);
    f.x2 = d_x2;
    f.nw = d_norm_w;
    f.eps = eps;
    f.res = d_res;
    const int r = tb::mv_launch(W_dev, qtype, M, K, d_x, d_y, static_cast<cudaStream_t>(stream), derr, nsm,
                                lim, &f);
    if (r) g_launches.fetch_add(1, std::memory_order_relaxed);
    return r;
}

int tb_cuda_dequant_dev(const void *W_dev, int qtype, int M, int K, float *d_out, int sem, void *stream)
{
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!ensure_init_locked(false)) return 0;
    }
    const int r = tb::dq_launch(W_dev, qtype, M, K, d_out, sem, static_cast<cudaStream_t>(stream));
    if (r) g_launches.fetch_add(1, std::memory_order_relaxed);
    return r;
}

int tb_cuda_last_error(void)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g.d_err) return 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return tb::ERR_RUNTIME;
    int e = 0;
    if (cudaMemcpy(&e, g.d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return tb::ERR_RUNTIME;
    cudaMemset(g.d_err, 0, sizeof(int));
    return e;
}

unsigned long long tb_cuda_launch_count(void) { return g_launches.load(); }

int tb_cuda_set_matvec_arith(int mode) { return tb::mv_set_arith(mode); }

int tb_cuda_get_matvec_arith(void) { return tb::mv_get_arith(); }

int tb_cuda_matvec_device_noalloc(const void *W_device, int qtype, int M, int K, const float *x_host,
                                  float *out_host)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!W_device || !x_host || !out_host || M <= 0 || K <= 0) return 0;
    const tb::Geom gg = tb::geom_of(qtype);
    if (!gg.block_weights || K % gg.block_weights) return 0;
    if (K > kNaMaxK || M > kNaMaxM) {
        fprintf(stderr, "[tb_cuda] matvec_device_noalloc: M=%d K=%d exceed the static buffers (M <= %d, K <= %d)\n",
                M, K, kNaMaxM, kNaMaxK);
        return 0;
    }
    const NaDev *d = na_device_locked();
    if (!d) return 0;
    const uint32_t lim = g.stream ? g.wait_limit : (1u << 22);
    const cudaStream_t st = nullptr;   // legacy default stream: no stream is created
    const size_t xb = static_cast<size_t>(K) * sizeof(float), yb = static_cast<size_t>(M) * sizeof(float);
    // the error word must start at zero; x and y are fully overwritten
    if (!cuda_ok(cudaMemsetAsync(d->err, 0, sizeof(int), st), "noalloc err clear")) return 0;
    if (!cuda_ok(cudaMemcpyAsync(d->x, x_host, xb, cudaMemcpyHostToDevice, st), "noalloc x H2D")) return 0;
    if (!tb::mv_launch(W_device, qtype, M, K, d->x, d->y, st, d->err, d->sms, lim)) return 0;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    int e = 0;
    if (!cuda_ok(cudaMemcpyAsync(out_host, d->y, yb, cudaMemcpyDeviceToHost, st), "noalloc y D2H")) return 0;
    if (!cuda_ok(cudaMemcpyAsync(&e, d->err, sizeof(int), cudaMemcpyDeviceToHost, st), "noalloc err D2H"))
        return 0;
    if (!cuda_ok(cudaStreamSynchronize(st), "noalloc sync")) return 0;
    if (e != 0) {
        fprintf(stderr, "[tb_cuda] matvec_device_noalloc: device error %d\n", e);
        return 0;
    }
    return 1;
}

}  // extern "C"
