// C ABI of libb200quant.so (declared in include/b200quant.h).
//
// Part 1 keeps the reference's exported names and signatures
// (engine/native_quant.cpp:705-768): host pointers in, host result out, with
// the copies and the kernel launch inside the call.  Part 2 is the
// device-pointer API used by the PyTorch host code.
#include "b200quant.h"
#include "common.cuh"
#include "ep.cuh"

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace b200q {
cudaError_t launch_dequant_f32(int type, const void *raw, float *out, long long nblocks, int num_sms, cudaStream_t st);
cudaError_t launch_dequant_bf16(int type, const void *raw, __nv_bfloat16 *out, long long nblocks, int num_sms,
                                cudaStream_t st);
cudaError_t launch_gemv(int type, const void *w, const float *x, float *y, long long ys_t, long long ys_r, int rows,
                        int cols, int tokens, int *err, int num_sms, cudaStream_t st);
void gemv_set_tuning(int stage_target_bytes, int stages, int rpg_max, int ctas_per_sm);
void gemv_set_mma(bool on);
void tc_gemm_set_pair(bool on);
int tc_gemm_pairs_used();
void gemv_mma_set_tuning(int spw, int stages, int ctas_per_sm);
cudaError_t launch_moe_router(const float *h, const float *wr, const float *bias, float *logits, int T, int E, int D,
                              cudaStream_t st);
cudaError_t launch_moe_topk(const float *logits, const float *sel_bias, int T, int E, int k, int renorm, int *ids,
                            float *wts, cudaStream_t st);
int moe_num_blocks(int T);
size_t moe_route_workspace_bytes(int T, int E, int D, int num_sms);
cudaError_t launch_moe_route(const float *h, const float *wr, const float *bias, const float *sel_bias, int T, int E,
                             int D, int k, int renorm, float *logits, int *ids, float *wts, float *ws,
                             size_t ws_bytes, int num_sms, cudaStream_t st, __nv_bfloat16 *hb = nullptr);
cudaError_t launch_moe_dispatch(const int *ids, const float *wts, int T, int k, int E, const float *h, int D,
                                int *block_counts, int *base, int *offsets, int *slot_of, int *token_of,
                                float *slot_w, __nv_bfloat16 *xperm, int *err, cudaStream_t st);
cudaError_t launch_moe_scatter_bf16(const __nv_bfloat16 *h, int T, const int *slot_of, int k, int S, int D,
                                    __nv_bfloat16 *out, int *err, cudaStream_t st);
cudaError_t launch_moe_combine(const void *out, bool out_bf16, long long n_rows, const int *slot_of,
                               const float *slot_w, int T, int k,
                               int D, float *y, cudaStream_t st);
cudaError_t launch_moe_dispatch_noalloc(const int *ids, const float *wts, int T, int k, int E, const float *h, int D,
                                        int *offsets, int *slot_of, int *token_of, float *slot_w,
                                        __nv_bfloat16 *xperm, cudaStream_t st);
int noalloc_dispatch_max();
cudaError_t noalloc_dispatch_take_error(int *code);
cudaError_t launch_tc_gemm(int wtype, const __nv_bfloat16 *x, long long x_rows, int k, const void *w,
                           long long w_row_bytes, int groups,
                               int w_rows_per_group, int up_offset, int n_feat, const int *row_off,
                               const int *group_w, int n_weight_groups, float *out, __nv_bfloat16 *out_bf16,
                               long long ld_out, const float *row_scale, __nv_bfloat16 *act, long long ld_act,
                               int *err, int num_sms, int max_ctas, cudaStream_t st, const EpDev *ep_ret,
                               bool out_t = false, const EpPush *push = nullptr);
cudaError_t ep_create(int G, int me, int E_loc, int D, long long cap_send, long long cap_recv, void **out);
cudaError_t ep_ipc_handle(void *ctx, void *handle64);
size_t ep_ipc_handle_bytes();
cudaError_t ep_open(void *ctx, const void *handles);
cudaError_t ep_destroy(void *ctx);
bool ep_is_open(void *ctx);
void *ep_recv_rows(void *ctx);
void *ep_ret_rows(void *ctx);
EpDev *ep_dev(void *ctx);
const int *ep_group_offsets(void *ctx);
long long ep_cap_recv(void *ctx);
long long ep_cap_send(void *ctx);
int ep_local_experts(void *ctx);
int ep_d_model(void *ctx);
cudaError_t launch_ep_counts(void *ctx, const int *offsets, uint32_t epoch, int *err, cudaStream_t st);
cudaError_t launch_ep_send(void *ctx, const void *h, bool h_bf16, const int *token_of, const int *offsets, int S, int T,
                           uint32_t epoch, int *err, int num_sms, cudaStream_t st);
cudaError_t launch_ep_wait(void *ctx, int which, uint32_t epoch, int *err, cudaStream_t st);
cudaError_t launch_ep_signal(void *ctx, uint32_t epoch, cudaStream_t st);
void ep_set_wait_ns(unsigned long long ns);

cudaError_t launch_silu_mul(const float *gu, int T, int F, float *out, long long ld_out, int num_sms, cudaStream_t st);
cudaError_t launch_f32_to_bf16(const float *x, long long n, __nv_bfloat16 *out, int num_sms, cudaStream_t st);
cudaError_t launch_gemv_grouped(int type, const void *w, long long w_group_stride, int n_groups, const int *grp_off,
                                const float *x, float *y, long long ys_t, int rows, int cols, int max_tokens,
                                int x_rows, int active_groups, long long row_stride, int *err, int num_sms,
                                cudaStream_t st);
int gemv_grouped_max_tokens(int type, int cols);
cudaError_t launch_dequant_row(int type, const void *raw, long long row_bytes, int cols, const int *row_idx, int rows,
                               int n, float *out, int *err, cudaStream_t st);
cudaError_t launch_add_rmsnorm(float *x, const float *delta, const float *w, int T, int D, float eps, float *h,
                               __nv_bfloat16 *hb, cudaStream_t st);
cudaError_t launch_rope_kv(float *qkv, int T, int H, int KV, int hd, int rotary, float base, const float *inv_freq,
                           int neox, const int *pos, float *kc, float *vc, int max_seq, int *err, int num_sms,
                           cudaStream_t st);
cudaError_t launch_qkv_bias_norm(float *qkv, int T, int H, int KV, int hd, const float *bias, const float *qn,
                                 const float *kn, float eps, cudaStream_t st);
cudaError_t launch_attn_prefill(const float *qkv, const float *kc, const float *vc, const int *pos, int T, int H,
                                int KV, int hd, int max_seq, int window, __nv_bfloat16 *out, int *err, cudaStream_t st);
size_t attn_prefill_tc_scratch_bytes(int T, int H, int KV, int hd, int max_seq);
cudaError_t launch_attn_prefill_tc(const float *qkv, const float *kc, const float *vc, const int *pos, int T, int H,
                                   int KV, int hd, int max_seq, void *scratch, size_t scratch_bytes,
                                   __nv_bfloat16 *out, int *err, int num_sms, cudaStream_t st);
size_t attn_scratch_floats(int H, int hd, int max_seq);
cudaError_t launch_attn_decode(const float *q, const float *kc, const float *vc, const int *pos, int H, int KV, int hd,
                               int max_seq, int window, float *part, float *out, cudaStream_t st);
cudaError_t launch_argmax(const float *logits, int V, int *token, int *pos, int *out_tokens, int max_tokens,
                          unsigned long long *key, int num_sms, cudaStream_t st);
cudaError_t launch_moe_gather_f32(const float *h, int T, const int *token_of, int S, int D, float *out, int *err,
                                  cudaStream_t st);
cudaError_t launch_moe_gather_bf16(const __nv_bfloat16 *h, int T, const int *token_of, int S, int D,
                                   __nv_bfloat16 *out, int *err, cudaStream_t st);
cudaError_t launch_zaya_router_prep(const float *x, const float *prev, const float *w_eda, const float *norm_w, int T,
                                    int R, float eps, float *state, float *out, cudaStream_t st);
cudaError_t launch_gelu(float *x, long long n, int num_sms, cudaStream_t st);
cudaError_t launch_copy_rows_range(const void *src, void *dst, const int *offsets, int g, int D, int max_rows,
                                   int num_sms, cudaStream_t st);

// Library-wide state shared with the other translation units.
std::recursive_mutex g_lock;
long long g_launches = 0;

static int g_status = 0;
static char g_msg[512] = "ok";

int set_status(int code, const char *fmt, ...)
{
    g_status = code;
    if (fmt) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
        va_end(ap);
    } else {
        snprintf(g_msg, sizeof(g_msg), "ok");
    }
    return code;
}
int cuda_status(cudaError_t e, const char *what)
{
    if (e == cudaSuccess) return set_status(B200Q_OK, nullptr);
    if (e == cudaErrorInvalidValue)
        return set_status(B200Q_EINVAL, "%s: unsupported shape or argument (%s)", what, cudaGetErrorString(e));
    return set_status(B200Q_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Per-device resources of the device-pointer API: SM count and the sticky
// error word that kernels set when a bounded wait or index check fails.
struct DevInfo {
    int sms = 0;
    int *err = nullptr;
};
static std::vector<DevInfo> g_devs;

int current_device_info(DevInfo **out)
{
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_status(B200Q_ENODEV, "no CUDA device: %s", cudaGetErrorString(e));
    if ((int)g_devs.size() <= dev) g_devs.resize(dev + 1);
    DevInfo &d = g_devs[dev];
    if (!d.err) {
        e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_status(e, "device query");
        e = cudaMalloc(&d.err, sizeof(int));
        if (e != cudaSuccess) return cuda_status(e, "error word");
        e = cudaMemset(d.err, 0, sizeof(int));
        if (e != cudaSuccess) return cuda_status(e, "error word");
    }
    *out = &d;
    return B200Q_OK;
}

// ---------------------------------------------------------------- Part 1
struct HostCtx {
    int device = -1;
    cudaStream_t stream = nullptr;
    void *w = nullptr;
    size_t wcap = 0;
    float *x = nullptr;
    size_t xcap = 0;
    float *y = nullptr;
    size_t ycap = 0;
    __nv_bfloat16 *xb = nullptr;   // bf16 activations of the tensor-core matmul
    size_t xbcap = 0;
    int *row_off = nullptr;        // device {0, tokens}: the one group of that matmul
    size_t row_off_cap = 0;
    int *herr = nullptr;   // pinned host copy of the error word
};
static HostCtx g_host;

struct Registered {
    const uint8_t *host;
    size_t n;
    uint8_t *dev;
};
static std::vector<Registered> g_reg;

static int host_init(int device)
{
    if (g_host.device == device && g_host.stream) return B200Q_OK;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return set_status(B200Q_ENODEV, "no CUDA device available");
    if (device < 0 || device >= n) return set_status(B200Q_EINVAL, "device %d out of range [0,%d)", device, n);
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
    if (g_host.stream && g_host.device != device) return set_status(B200Q_EINVAL, "library already bound to device %d", g_host.device);
    e = cudaStreamCreateWithFlags(&g_host.stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_status(e, "stream");
    e = cudaMallocHost(&g_host.herr, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "pinned error word");
    g_host.device = device;
    return B200Q_OK;
}

int grow(void **p, size_t *cap, size_t need);
int grow(void **p, size_t *cap, size_t need)
{
    if (need <= *cap) return B200Q_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    const size_t sz = need + need / 4 + 256;
    cudaError_t e = cudaMalloc(p, sz);
    if (e != cudaSuccess) return cuda_status(e, "device buffer");
    *cap = sz;
    return B200Q_OK;
}

static const uint8_t *lookup_registered(const uint8_t *raw, size_t n)
{
    for (const Registered &r : g_reg)
        if (raw >= r.host && raw + n <= r.host + r.n) return r.dev + (raw - r.host);
    return nullptr;
}

// Batched Part-1 calls (the reference's prefill path: decoded_matmul_row,
// engine/native_quant.cpp:620-703) with at least this many tokens run on the
// tensor cores (bf16 operands, f32 accumulation) when the type and shape allow
// it; smaller batches, other types and other shapes take the f32 GEMV.
// 0 keeps every call on the GEMV.
static int g_tc_min_tokens = 32;

// Q4_K/Q5_K/Q6_K/Q8_0/Q4_0 weights whose packed rows are whole 16-byte units
// (the GEMM streams them with TMA), a multiple of 128 rows and of 64 columns.
static bool tc_matmul_shape_ok(int type, const void *wdev, int rows, int cols)
{
    if (type != T_Q4_K && type != T_Q5_K && type != T_Q6_K && type != T_Q8_0 && type != T_Q4_0) return false;
    if (rows % 128 || cols % 64 || (reinterpret_cast<uintptr_t>(wdev) & 15)) return false;
    const long long rb = (long long)(cols / type_vals(type)) * type_bytes(type);
    return rb % 16 == 0;
}

// One Part-1 call: upload, launch, download, wait, report.
static void host_call(int type, const uint8_t *raw, const float *x, float *out, int rows, int cols, int tokens,
                      bool matmul)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    const int vals = type_vals(type), bytes = type_bytes(type);
    if (!raw || !x || !out) { set_status(B200Q_EINVAL, "null pointer"); return; }
    if (!bytes || rows < 1 || tokens < 1 || cols < vals || cols % vals) {
        set_status(B200Q_EINVAL, "invalid shape rows=%d cols=%d tokens=%d for type %d", rows, cols, tokens, type);
        return;
    }
    if (g_host.device < 0 && host_init(0) != B200Q_OK) return;
    cudaSetDevice(g_host.device);
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return;
    const size_t wbytes = (size_t)rows * (cols / vals) * bytes;
    const size_t xbytes = (size_t)tokens * cols * sizeof(float);
    const size_t ybytes = (size_t)tokens * rows * sizeof(float);
    cudaStream_t st = g_host.stream;
    const uint8_t *wdev = lookup_registered(raw, wbytes);
    if (!wdev) {
        if (grow(&g_host.w, &g_host.wcap, wbytes) != B200Q_OK) return;
        cudaError_t e = cudaMemcpyAsync(g_host.w, raw, wbytes, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) { cuda_status(e, "weight upload"); return; }
        wdev = static_cast<const uint8_t *>(g_host.w);
    }
    if (grow((void **)&g_host.x, &g_host.xcap, xbytes) != B200Q_OK) return;
    if (grow((void **)&g_host.y, &g_host.ycap, ybytes) != B200Q_OK) return;
    cudaError_t e = cudaMemcpyAsync(g_host.x, x, xbytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) { cuda_status(e, "input upload"); return; }
    // Reference output layout: matvec [rows]; matmul [rows][tokens]
    // (engine/native_quant.py:148-156).
    if (matmul && g_tc_min_tokens > 0 && tokens >= g_tc_min_tokens && tc_matmul_shape_ok(type, wdev, rows, cols)) {
        const size_t xbbytes = (size_t)tokens * cols * sizeof(__nv_bfloat16);
        if (grow((void **)&g_host.xb, &g_host.xbcap, xbbytes) != B200Q_OK) return;
        if (grow((void **)&g_host.row_off, &g_host.row_off_cap, 2 * sizeof(int)) != B200Q_OK) return;
        const int off[2] = {0, tokens};
        e = cudaMemcpyAsync(g_host.row_off, off, sizeof(off), cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = launch_f32_to_bf16(g_host.x, (long long)tokens * cols, g_host.xb, di->sms, st);
        if (e == cudaSuccess)
            e = launch_tc_gemm(type, g_host.xb, tokens, cols, wdev, 0, 1, rows, -1, rows, g_host.row_off, nullptr, 1,
                               g_host.y, nullptr, tokens, nullptr, nullptr, 0, di->err, di->sms, 0, st, nullptr,
                               true);
        g_launches += 2;
        if (e != cudaSuccess) { cuda_status(e, "tensor-core matmul launch"); return; }
    } else {
        const long long ys_t = matmul ? 1 : rows, ys_r = matmul ? tokens : 1;
        e = launch_gemv(type, wdev, g_host.x, g_host.y, ys_t, ys_r, rows, cols, tokens, di->err, di->sms, st);
        ++g_launches;
        if (e != cudaSuccess) { cuda_status(e, "gemv launch"); return; }
    }
    e = cudaMemcpyAsync(out, g_host.y, ybytes, cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) { cuda_status(e, "output download"); return; }
    e = cudaMemcpyAsync(g_host.herr, di->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { cuda_status(e, "synchronize"); return; }
    if (*g_host.herr) {
        const int code = *g_host.herr;
        cudaMemsetAsync(di->err, 0, sizeof(int), st);
        cudaStreamSynchronize(st);
        set_status(code == ERR_WAIT_TIMEOUT ? B200Q_ETIMEOUT : B200Q_EINDEX, "kernel reported error %d", code);
        return;
    }
    set_status(B200Q_OK, nullptr);
}

} // namespace b200q

using namespace b200q;

#define B200Q_API extern "C" __attribute__((visibility("default")))

B200Q_API void localai_q8_0_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads)
{
    (void)threads;
    host_call(T_Q8_0, raw, x, out, rows, cols, 1, false);
}
B200Q_API void localai_q4_0_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads)
{
    (void)threads;
    host_call(T_Q4_0, raw, x, out, rows, cols, 1, false);
}
B200Q_API void localai_q4k_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads)
{
    (void)threads;
    host_call(T_Q4_K, raw, x, out, rows, cols, 1, false);
}
B200Q_API void localai_q5k_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads)
{
    (void)threads;
    host_call(T_Q5_K, raw, x, out, rows, cols, 1, false);
}
B200Q_API void localai_q6k_matvec(const uint8_t *raw, const float *x, float *out, int rows, int cols, int threads)
{
    (void)threads;
    host_call(T_Q6_K, raw, x, out, rows, cols, 1, false);
}
B200Q_API void localai_q8_0_matmul(const uint8_t *raw, const float *v, float *out, int rows, int cols, int tokens,
                                   int threads)
{
    (void)threads;
    host_call(T_Q8_0, raw, v, out, rows, cols, tokens, true);
}
B200Q_API void localai_q4_0_matmul(const uint8_t *raw, const float *v, float *out, int rows, int cols, int tokens,
                                   int threads)
{
    (void)threads;
    host_call(T_Q4_0, raw, v, out, rows, cols, tokens, true);
}
B200Q_API void localai_q4k_matmul(const uint8_t *raw, const float *v, float *out, int rows, int cols, int tokens,
                                  int threads)
{
    (void)threads;
    host_call(T_Q4_K, raw, v, out, rows, cols, tokens, true);
}
B200Q_API void localai_q5k_matmul(const uint8_t *raw, const float *v, float *out, int rows, int cols, int tokens,
                                  int threads)
{
    (void)threads;
    host_call(T_Q5_K, raw, v, out, rows, cols, tokens, true);
}
B200Q_API void localai_q6k_matmul(const uint8_t *raw, const float *v, float *out, int rows, int cols, int tokens,
                                  int threads)
{
    (void)threads;
    host_call(T_Q6_K, raw, v, out, rows, cols, tokens, true);
}

B200Q_API int b200q_matmul_tensor_core_min_tokens(int tokens)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    const int prev = g_tc_min_tokens;
    if (tokens >= 0) g_tc_min_tokens = tokens;
    return prev;
}

B200Q_API int b200q_last_status(void) { return g_status; }
B200Q_API const char *b200q_last_error(void) { return g_msg; }

B200Q_API int b200q_init(int device)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    return host_init(device) == B200Q_OK ? set_status(B200Q_OK, nullptr) : g_status;
}

B200Q_API int b200q_register_host(const void *ptr, size_t nbytes)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ptr || !nbytes) return set_status(B200Q_EINVAL, "register: null or empty range");
    if (g_host.device < 0 && host_init(0) != B200Q_OK) return g_status;
    cudaSetDevice(g_host.device);
    const uint8_t *p = static_cast<const uint8_t *>(ptr);
    for (const Registered &r : g_reg)
        if (r.host == p && r.n == nbytes) return set_status(B200Q_OK, nullptr);
    uint8_t *dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, nbytes + 64);
    if (e != cudaSuccess) return cuda_status(e, "register: cudaMalloc");
    e = cudaMemcpy(dev, p, nbytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(dev);
        return cuda_status(e, "register: upload");
    }
    g_reg.push_back({p, nbytes, dev});
    return set_status(B200Q_OK, nullptr);
}

B200Q_API int b200q_unregister_host(const void *ptr)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    for (size_t i = 0; i < g_reg.size(); ++i)
        if (g_reg[i].host == ptr) {
            cudaFree(g_reg[i].dev);
            g_reg.erase(g_reg.begin() + i);
            return set_status(B200Q_OK, nullptr);
        }
    return set_status(B200Q_EINVAL, "unregister: pointer not registered");
}

B200Q_API int b200q_registry_clear(void)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    for (Registered &r : g_reg) cudaFree(r.dev);
    g_reg.clear();
    return set_status(B200Q_OK, nullptr);
}

B200Q_API void *b200q_registered_device_ptr(const void *host_ptr)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    return (void *)lookup_registered(static_cast<const uint8_t *>(host_ptr), 1);
}

B200Q_API int b200q_dequant_f32_dev(int ggml_type, const void *w, float *out, long long nblocks, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!w || !out || nblocks < 0 || !type_bytes(ggml_type)) return set_status(B200Q_EINVAL, "dequant: bad argument");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_dequant_f32(ggml_type, w, out, nblocks, di->sms, (cudaStream_t)stream), "dequant");
}

B200Q_API int b200q_dequant_bf16_dev(int ggml_type, const void *w, void *out, long long nblocks, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!w || !out || nblocks < 0 || !type_bytes(ggml_type)) return set_status(B200Q_EINVAL, "dequant: bad argument");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_dequant_bf16(ggml_type, w, static_cast<__nv_bfloat16 *>(out), nblocks, di->sms,
                                           (cudaStream_t)stream),
                       "dequant");
}

B200Q_API int b200q_gemv_dev(int ggml_type, const void *w, const float *x, float *y, int rows, int cols, int tokens,
                             long long ys_t, long long ys_r, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!w || !x || !y) return set_status(B200Q_EINVAL, "gemv: null pointer");
    if ((reinterpret_cast<uintptr_t>(w) & 1) || (reinterpret_cast<uintptr_t>(x) & 15))
        return set_status(B200Q_EINVAL, "gemv: weights must be 2-byte and x 16-byte aligned");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_gemv(ggml_type, w, x, y, ys_t, ys_r, rows, cols, tokens, di->err, di->sms,
                                   (cudaStream_t)stream),
                       "gemv");
}

B200Q_API int b200q_gemm_q4k_dev(const void *x_bf16, long long x_rows, int k, const void *w, int groups,
                                 int w_rows_per_group, int up_offset, int n_feat, const int *row_off,
                                 const int *group_w, int n_weight_groups, void *out, int out_is_bf16,
                                 long long ld_out, const float *row_scale, void *act_bf16, long long ld_act,
                                 int max_ctas, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!x_bf16 || !w || !row_off) return set_status(B200Q_EINVAL, "gemm: null pointer");
    if (up_offset >= 0 ? !act_bf16 : !out) return set_status(B200Q_EINVAL, "gemm: missing output");
    if (group_w && n_weight_groups < 1) return set_status(B200Q_EINVAL, "gemm: n_weight_groups must be >= 1");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_tc_gemm(T_Q4_K, static_cast<const __nv_bfloat16 *>(x_bf16), x_rows, k, w, 0, groups,
                                          w_rows_per_group, up_offset, n_feat, row_off, group_w, n_weight_groups,
                                          out_is_bf16 ? nullptr : static_cast<float *>(out),
                                          out_is_bf16 ? static_cast<__nv_bfloat16 *>(out) : nullptr, ld_out,
                                          row_scale, static_cast<__nv_bfloat16 *>(act_bf16), ld_act, di->err,
                                          di->sms, max_ctas, (cudaStream_t)stream, nullptr),
                       "gemm");
}

B200Q_API int b200q_gemm_dev(int ggml_type, const void *x_bf16, long long x_rows, int k, const void *w,
                             long long w_row_bytes, int groups, int w_rows_per_group, int up_offset, int n_feat,
                             const int *row_off, const int *group_w, int n_weight_groups, void *out, int out_is_bf16,
                             long long ld_out, const float *row_scale, void *act_bf16, long long ld_act, int max_ctas,
                             void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!x_bf16 || !w || !row_off) return set_status(B200Q_EINVAL, "gemm: null pointer");
    if (up_offset >= 0 ? !act_bf16 : !out) return set_status(B200Q_EINVAL, "gemm: missing output");
    if (group_w && n_weight_groups < 1) return set_status(B200Q_EINVAL, "gemm: n_weight_groups must be >= 1");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_tc_gemm(ggml_type, static_cast<const __nv_bfloat16 *>(x_bf16), x_rows, k, w,
                                      w_row_bytes, groups, w_rows_per_group, up_offset, n_feat, row_off, group_w,
                                      n_weight_groups, out_is_bf16 ? nullptr : static_cast<float *>(out),
                                      out_is_bf16 ? static_cast<__nv_bfloat16 *>(out) : nullptr, ld_out, row_scale,
                                      static_cast<__nv_bfloat16 *>(act_bf16), ld_act, di->err, di->sms, max_ctas,
                                      (cudaStream_t)stream, nullptr),
                       "gemm");
}

B200Q_API int b200q_zaya_router_prep_dev(const float *x, const float *prev, const float *w_eda, const float *norm_w,
                                         int T, int R, float eps, float *state, float *out, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!x || !norm_w || !state || !out) return set_status(B200Q_EINVAL, "zaya_router_prep: null pointer");
    ++g_launches;
    return cuda_status(launch_zaya_router_prep(x, prev, w_eda, norm_w, T, R, eps, state, out, (cudaStream_t)stream),
                       "zaya_router_prep");
}

B200Q_API int b200q_gelu_dev(float *x, long long n, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!x) return set_status(B200Q_EINVAL, "gelu: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_gelu(x, n, di->sms, (cudaStream_t)stream), "gelu");
}

B200Q_API int b200q_copy_rows_range_dev(const void *src_bf16, void *dst_bf16, const int *offsets, int group, int D,
                                        int max_rows, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!src_bf16 || !dst_bf16 || !offsets) return set_status(B200Q_EINVAL, "copy_rows_range: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_copy_rows_range(src_bf16, dst_bf16, offsets, group, D, max_rows, di->sms,
                                              (cudaStream_t)stream),
                       "copy_rows_range");
}

B200Q_API int b200q_silu_mul_dev(const float *gate_up, int T, int F, float *out, long long ld_out, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!gate_up || !out) return set_status(B200Q_EINVAL, "silu_mul: null pointer");
    if (ld_out < F) return set_status(B200Q_EINVAL, "silu_mul: ld_out < F");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_silu_mul(gate_up, T, F, out, ld_out, di->sms, (cudaStream_t)stream), "silu_mul");
}

B200Q_API int b200q_gemv_grouped_max_tokens(int ggml_type, int cols) { return gemv_grouped_max_tokens(ggml_type, cols); }

B200Q_API int b200q_gemv_grouped_dev(int ggml_type, const void *w, long long w_group_stride, long long w_row_bytes,
                                     int n_groups, const int *grp_off, const float *x, float *y, long long ys_t,
                                     int rows, int cols, int max_tokens, int x_rows, int active_groups, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!w || !x || !y || !grp_off) return set_status(B200Q_EINVAL, "gemv_grouped: null pointer");
    if ((reinterpret_cast<uintptr_t>(w) & 1) || (reinterpret_cast<uintptr_t>(x) & 15) || (w_group_stride & 1))
        return set_status(B200Q_EINVAL, "gemv_grouped: weights must be 2-byte and x 16-byte aligned");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    if (w_row_bytes & 1) return set_status(B200Q_EINVAL, "gemv_grouped: odd row stride");
    return cuda_status(launch_gemv_grouped(ggml_type, w, w_group_stride, n_groups, grp_off, x, y, ys_t, rows, cols,
                                           max_tokens, x_rows, active_groups, w_row_bytes, di->err, di->sms,
                                           (cudaStream_t)stream),
                       "gemv_grouped");
}

B200Q_API int b200q_moe_gather_f32_dev(const float *h, int h_rows, const int *token_of, int S, int D, float *out,
                                       void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!h || !token_of || !out) return set_status(B200Q_EINVAL, "gather_f32: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_moe_gather_f32(h, h_rows, token_of, S, D, out, di->err, (cudaStream_t)stream),
                       "gather_f32");
}

B200Q_API int b200q_moe_gather_bf16_dev(const void *h_bf16, int h_rows, const int *token_of, int S, int D, void *out,
                                        void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!h_bf16 || !token_of || !out) return set_status(B200Q_EINVAL, "gather_bf16: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_moe_gather_bf16(static_cast<const __nv_bfloat16 *>(h_bf16), h_rows, token_of, S, D,
                                              static_cast<__nv_bfloat16 *>(out), di->err, (cudaStream_t)stream),
                       "gather_bf16");
}

B200Q_API int b200q_moe_scatter_bf16_dev(const void *h_bf16, int T, const int *slot_of, int k, int S, int D, void *out,
                                         void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!h_bf16 || !slot_of || !out) return set_status(B200Q_EINVAL, "scatter_bf16: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_moe_scatter_bf16(static_cast<const __nv_bfloat16 *>(h_bf16), T, slot_of, k, S, D,
                                               static_cast<__nv_bfloat16 *>(out), di->err, (cudaStream_t)stream),
                       "scatter_bf16");
}

B200Q_API int b200q_moe_router_dev(const float *h, const float *wr, const float *bias, float *logits, int T, int E,
                                   int D, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!h || !wr || !logits) return set_status(B200Q_EINVAL, "router: null pointer");
    ++g_launches;
    return cuda_status(launch_moe_router(h, wr, bias, logits, T, E, D, (cudaStream_t)stream), "router");
}

B200Q_API int b200q_moe_topk_dev(const float *logits, const float *sel_bias, int T, int E, int k, int renormalize,
                                 int *ids, float *w, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!logits || !ids || !w) return set_status(B200Q_EINVAL, "topk: null pointer");
    ++g_launches;
    return cuda_status(launch_moe_topk(logits, sel_bias, T, E, k, renormalize, ids, w, (cudaStream_t)stream), "topk");
}

B200Q_API int b200q_moe_num_blocks(int T) { return moe_num_blocks(T); }

B200Q_API size_t b200q_moe_route_workspace_bytes(int T, int E, int D)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return 0;
    return moe_route_workspace_bytes(T, E, D, di->sms);
}

B200Q_API int b200q_moe_route_dev(const float *h, const float *wr, const float *bias, const float *sel_bias, int T,
                                  int E, int D, int k, int renormalize, float *logits, int *ids, float *w,
                                  void *workspace, size_t workspace_bytes, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!h || !wr || !logits || !ids || !w) return set_status(B200Q_EINVAL, "route: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    g_launches += 2;
    return cuda_status(launch_moe_route(h, wr, bias, sel_bias, T, E, D, k, renormalize, logits, ids, w,
                                        static_cast<float *>(workspace), workspace_bytes, di->sms,
                                        (cudaStream_t)stream),
                       "route");
}

B200Q_API int b200q_moe_route_bf16_dev(const float *h, const float *wr, const float *bias, const float *sel_bias,
                                       int T, int E, int D, int k, int renormalize, float *logits, int *ids, float *w,
                                       void *workspace, size_t workspace_bytes, void *h_bf16, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!h || !wr || !logits || !ids || !w || !h_bf16) return set_status(B200Q_EINVAL, "route: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    g_launches += 2;
    return cuda_status(launch_moe_route(h, wr, bias, sel_bias, T, E, D, k, renormalize, logits, ids, w,
                                        static_cast<float *>(workspace), workspace_bytes, di->sms,
                                        (cudaStream_t)stream, static_cast<__nv_bfloat16 *>(h_bf16)),
                       "route");
}

B200Q_API int b200q_moe_dispatch_dev(const int *ids, const float *w, int T, int k, int E, const float *h, int D,
                                     int *block_counts, int *base, int *offsets, int *slot_of, int *token_of,
                                     float *slot_w, void *xperm_bf16, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ids || !w || !block_counts || !base || !offsets || !slot_of || !token_of || !slot_w || (xperm_bf16 && !h))
        return set_status(B200Q_EINVAL, "dispatch: null pointer");
    if (E > 1024) return set_status(B200Q_EINVAL, "dispatch: at most 1024 experts");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    g_launches += xperm_bf16 ? 4 : 3;
    return cuda_status(launch_moe_dispatch(ids, w, T, k, E, h, D, block_counts, base, offsets, slot_of, token_of,
                                           slot_w, static_cast<__nv_bfloat16 *>(xperm_bf16), di->err,
                                           (cudaStream_t)stream),
                       "dispatch");
}

// Allocation-free variant of b200q_moe_dispatch_dev: scratch in a file-scope
// device array (see moe.cu); no cudaMalloc, cudaFree or allocating library call.
B200Q_API int b200q_moe_dispatch_noalloc_dev(const int *ids, const float *w, int T, int k, int E, const float *h,
                                             int D, int *offsets, int *slot_of, int *token_of, float *slot_w,
                                             void *xperm_bf16, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ids || !w || !offsets || !slot_of || !token_of || !slot_w || (xperm_bf16 && !h))
        return set_status(B200Q_EINVAL, "dispatch_noalloc: null pointer");
    if (T < 1 || k < 1 || E < 1 || E > 1024)
        return set_status(B200Q_EINVAL, "dispatch_noalloc: invalid T=%d k=%d E=%d", T, k, E);
    if ((long long)moe_num_blocks(T) * E > noalloc_dispatch_max())
        return set_status(B200Q_EINVAL,
                          "dispatch_noalloc: ceil(T/256)*E = %lld exceeds the static scratch limit of %d entries",
                          (long long)moe_num_blocks(T) * E, noalloc_dispatch_max());
    g_launches += xperm_bf16 ? 4 : 3;
    return cuda_status(launch_moe_dispatch_noalloc(ids, w, T, k, E, h, D, offsets, slot_of, token_of, slot_w,
                                                   static_cast<__nv_bfloat16 *>(xperm_bf16), (cudaStream_t)stream),
                       "dispatch_noalloc");
}

B200Q_API int b200q_moe_combine_dev(const void *out, int out_is_bf16, const int *slot_of, const float *slot_w, int T,
                                    int k, int D, float *y, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!out || !slot_of || !y) return set_status(B200Q_EINVAL, "combine: null pointer");
    ++g_launches;
    return cuda_status(launch_moe_combine(out, out_is_bf16 != 0, (long long)T * k, slot_of, slot_w, T, k, D, y,
                                          (cudaStream_t)stream),
                       "combine");
}

B200Q_API int b200q_check_device_error(void)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_status(e, "synchronize");
    int v = 0;
    e = cudaMemcpy(&v, di->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_status(e, "error word read");
    if (v) cudaMemset(di->err, 0, sizeof(int));
    // the allocation-free dispatch keeps its own error word in static device memory
    int v2 = 0;
    e = noalloc_dispatch_take_error(&v2);
    if (e != cudaSuccess) return cuda_status(e, "error word read");
    set_status(B200Q_OK, nullptr);
    return v ? v : v2;
}

B200Q_API void b200q_gemv_tuning(int stage_bytes, int stages, int rows_per_group, int ctas_per_sm)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    gemv_set_tuning(stage_bytes, stages, rows_per_group, ctas_per_sm);
}

B200Q_API void b200q_gemv_mma_tuning(int enable, int sb_per_warp, int stages, int ctas_per_sm)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (enable >= 0) gemv_set_mma(enable != 0);
    gemv_mma_set_tuning(sb_per_warp, stages, ctas_per_sm);
}

B200Q_API int b200q_gemm_pair_mode(int on)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (on >= 0) tc_gemm_set_pair(on != 0);
    return tc_gemm_pairs_used();
}

B200Q_API long long b200q_launch_count(void) { return g_launches; }

// ---------------------------------------------------------------- expert-parallel exchange over peer memory
B200Q_API int b200q_ep_create(int world, int rank, int local_experts, int d_model, long long max_send_rows,
                              long long max_recv_rows, void **ep)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep) return set_status(B200Q_EINVAL, "ep_create: null output");
    return cuda_status(ep_create(world, rank, local_experts, d_model, max_send_rows, max_recv_rows, ep), "ep_create");
}

B200Q_API size_t b200q_ep_handle_bytes(void) { return ep_ipc_handle_bytes(); }

B200Q_API void b200q_ep_set_wait_limit_ns(unsigned long long ns)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    ep_set_wait_ns(ns);
}

B200Q_API int b200q_ep_handle(void *ep, void *handle)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !handle) return set_status(B200Q_EINVAL, "ep_handle: null pointer");
    return cuda_status(ep_ipc_handle(ep, handle), "ep_handle");
}

B200Q_API int b200q_ep_open(void *ep, const void *handles)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !handles) return set_status(B200Q_EINVAL, "ep_open: null pointer");
    return cuda_status(ep_open(ep, handles), "ep_open");
}

B200Q_API int b200q_ep_destroy(void *ep)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep) return set_status(B200Q_EINVAL, "ep_destroy: null pointer");
    return cuda_status(ep_destroy(ep), "ep_destroy");
}

B200Q_API void *b200q_ep_recv_rows(void *ep) { return ep ? ep_recv_rows(ep) : nullptr; }
B200Q_API void *b200q_ep_return_rows(void *ep) { return ep ? ep_ret_rows(ep) : nullptr; }
B200Q_API const int *b200q_ep_group_offsets(void *ep) { return ep ? ep_group_offsets(ep) : nullptr; }

B200Q_API int b200q_ep_exchange_counts_dev(void *ep, const int *offsets, unsigned int epoch, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !offsets) return set_status(B200Q_EINVAL, "ep_exchange_counts: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_ep_counts(ep, offsets, epoch, di->err, (cudaStream_t)stream), "ep_exchange_counts");
}

B200Q_API int b200q_ep_send_rows_dev(void *ep, const float *h, int T, const int *token_of, const int *offsets,
                                     int slots, unsigned int epoch, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !h || !token_of || !offsets) return set_status(B200Q_EINVAL, "ep_send_rows: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_ep_send(ep, h, false, token_of, offsets, slots, T, epoch, di->err, di->sms,
                                      (cudaStream_t)stream),
                       "ep_send_rows");
}

B200Q_API int b200q_ep_send_rows_bf16_dev(void *ep, const void *h_bf16, int T, const int *token_of,
                                          const int *offsets, int slots, unsigned int epoch, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !h_bf16 || !token_of || !offsets) return set_status(B200Q_EINVAL, "ep_send_rows: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_ep_send(ep, h_bf16, true, token_of, offsets, slots, T, epoch, di->err, di->sms,
                                      (cudaStream_t)stream),
                       "ep_send_rows");
}

B200Q_API int b200q_ep_experts_dev(void *ep, int ggml_type, const void *gate_up, long long gate_up_row_bytes,
                                   const void *down, long long down_row_bytes, int d_ff, void *act,
                                   unsigned int epoch, int max_ctas, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !gate_up || !down || !act) return set_status(B200Q_EINVAL, "ep_experts: null pointer");
    if (d_ff < 64 || d_ff % 64) return set_status(B200Q_EINVAL, "ep_experts: d_ff must be a multiple of 64");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    const cudaStream_t st = (cudaStream_t)stream;
    const int El = ep_local_experts(ep), D = ep_d_model(ep);
    const long long cap = ep_cap_recv(ep);
    const int *grp = ep_group_offsets(ep);
    cudaError_t e = launch_ep_wait(ep, 1, epoch, di->err, st);
    if (e == cudaSuccess)
        e = launch_tc_gemm(ggml_type, static_cast<const __nv_bfloat16 *>(ep_recv_rows(ep)), cap, D, gate_up,
                           gate_up_row_bytes, El, 2 * d_ff,
                               d_ff, d_ff, grp, nullptr, El, nullptr, nullptr, 0, nullptr,
                               static_cast<__nv_bfloat16 *>(act), d_ff, di->err, di->sms, max_ctas, st, nullptr);
    if (e == cudaSuccess)
        e = launch_tc_gemm(ggml_type, static_cast<const __nv_bfloat16 *>(act), cap, d_ff, down, down_row_bytes, El, D,
                           -1, D, grp,
                               nullptr, El, nullptr, nullptr, D, nullptr, nullptr, 0, di->err, di->sms, max_ctas, st,
                               ep_dev(ep));
    if (e == cudaSuccess) e = launch_ep_signal(ep, epoch, st);
    g_launches += 4;
    return cuda_status(e, "ep_experts");
}

B200Q_API int b200q_ep_dispatch_experts_dev(void *ep, int ggml_type, const void *gate_up, long long gate_up_row_bytes,
                                            const void *down, long long down_row_bytes, int d_ff, void *act,
                                            const void *h_bf16, int T, const int *token_of, const int *offsets,
                                            int slots, unsigned int epoch, int max_ctas, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !gate_up || !down || !act || !h_bf16 || !token_of || !offsets)
        return set_status(B200Q_EINVAL, "ep_dispatch_experts: null pointer");
    if (d_ff < 64 || d_ff % 64) return set_status(B200Q_EINVAL, "ep_dispatch_experts: d_ff must be a multiple of 64");
    if (T < 0 || slots < 0 || (long long)slots > ep_cap_send(ep))
        return set_status(B200Q_EINVAL, "ep_dispatch_experts: more slots than max_send_rows");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    const cudaStream_t st = (cudaStream_t)stream;
    const int El = ep_local_experts(ep), D = ep_d_model(ep);
    const long long cap = ep_cap_recv(ep);
    const int *grp = ep_group_offsets(ep);
    EpPush push;
    push.ep = ep_dev(ep);
    push.h = static_cast<const __nv_bfloat16 *>(h_bf16);
    push.token_of = token_of;
    push.offsets = offsets;
    push.S = slots;
    push.T = T;
    push.epoch = epoch;
    push.wait_ns = ep_wait_ns();
    cudaError_t e = launch_tc_gemm(ggml_type, static_cast<const __nv_bfloat16 *>(ep_recv_rows(ep)), cap, D, gate_up,
                                   gate_up_row_bytes, El, 2 * d_ff, d_ff, d_ff, grp, nullptr, El, nullptr, nullptr, 0,
                                   nullptr, static_cast<__nv_bfloat16 *>(act), d_ff, di->err, di->sms, max_ctas, st,
                                   nullptr, false, &push);
    if (e == cudaSuccess)
        e = launch_tc_gemm(ggml_type, static_cast<const __nv_bfloat16 *>(act), cap, d_ff, down, down_row_bytes, El, D,
                           -1, D, grp, nullptr, El, nullptr, nullptr, D, nullptr, nullptr, 0, di->err, di->sms,
                           max_ctas, st, ep_dev(ep));
    if (e == cudaSuccess) e = launch_ep_signal(ep, epoch, st);
    g_launches += 3;
    return cuda_status(e, "ep_dispatch_experts");
}

B200Q_API int b200q_ep_combine_dev(void *ep, const int *slot_of, const float *slot_w, int T, int k, float *y,
                                   unsigned int epoch, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!ep || !slot_of || !slot_w || !y) return set_status(B200Q_EINVAL, "ep_combine: null pointer");
    if ((long long)T * k > ep_cap_send(ep)) return set_status(B200Q_EINVAL, "ep_combine: more slots than max_send_rows");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    const cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = launch_ep_wait(ep, 2, epoch, di->err, st);
    if (e == cudaSuccess)
        e = launch_moe_combine(ep_ret_rows(ep), true, ep_cap_send(ep), slot_of, slot_w, T, k, ep_d_model(ep), y, st);
    g_launches += 2;
    return cuda_status(e, "ep_combine");
}

// ---------------------------------------------------------------- decode step (Llama)
B200Q_API int b200q_dequant_row_dev(int ggml_type, const void *raw, long long row_bytes, int cols, const int *row_idx,
                                    int rows, int n, float *out, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!raw || !row_idx || !out) return set_status(B200Q_EINVAL, "dequant_row: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_dequant_row(ggml_type, raw, row_bytes, cols, row_idx, rows, n, out, di->err,
                                          (cudaStream_t)stream),
                       "dequant_row");
}

B200Q_API int b200q_add_rmsnorm_dev(float *x, const float *delta, const float *w, int T, int D, float eps, float *h,
                                    void *h_bf16, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!x || !w || (!h && !h_bf16)) return set_status(B200Q_EINVAL, "add_rmsnorm: null pointer");
    ++g_launches;
    return cuda_status(launch_add_rmsnorm(x, delta, w, T, D, eps, h, static_cast<__nv_bfloat16 *>(h_bf16),
                                          (cudaStream_t)stream),
                       "add_rmsnorm");
}

B200Q_API int b200q_rope_kv_dev(float *qkv, int T, int H, int KV, int hd, int rotary, float base, const int *pos,
                                float *k_cache, float *v_cache, int max_seq, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!qkv || !pos || !k_cache || !v_cache) return set_status(B200Q_EINVAL, "rope_kv: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_rope_kv(qkv, T, H, KV, hd, rotary, base, nullptr, 0, pos, k_cache, v_cache, max_seq,
                                      di->err, di->sms, (cudaStream_t)stream),
                       "rope_kv");
}

B200Q_API int b200q_rope_kv_ex_dev(float *qkv, int T, int H, int KV, int hd, int rotary, float base,
                                   const float *inv_freq, int neox, const int *pos, float *k_cache, float *v_cache,
                                   int max_seq, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!qkv || !pos || !k_cache || !v_cache) return set_status(B200Q_EINVAL, "rope_kv_ex: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_rope_kv(qkv, T, H, KV, hd, rotary, base, inv_freq, neox, pos, k_cache, v_cache, max_seq,
                                      di->err, di->sms, (cudaStream_t)stream),
                       "rope_kv_ex");
}

B200Q_API int b200q_qkv_bias_norm_dev(float *qkv, int T, int H, int KV, int hd, const float *bias, const float *q_norm,
                                      const float *k_norm, float eps, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!qkv) return set_status(B200Q_EINVAL, "qkv_bias_norm: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_qkv_bias_norm(qkv, T, H, KV, hd, bias, q_norm, k_norm, eps, (cudaStream_t)stream),
                       "qkv_bias_norm");
}

B200Q_API size_t b200q_attn_decode_scratch_floats(int H, int hd, int max_seq)
{
    return attn_scratch_floats(H, hd, max_seq);
}

B200Q_API int b200q_attn_decode_dev(const float *q, const float *k_cache, const float *v_cache, const int *pos, int H,
                                    int KV, int hd, int max_seq, float *scratch, float *out, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!q || !k_cache || !v_cache || !pos || !scratch || !out) return set_status(B200Q_EINVAL, "attn: null pointer");
    g_launches += 2;
    return cuda_status(launch_attn_decode(q, k_cache, v_cache, pos, H, KV, hd, max_seq, 0, scratch, out,
                                          (cudaStream_t)stream),
                       "attn_decode");
}

B200Q_API int b200q_attn_decode_ex_dev(const float *q, const float *k_cache, const float *v_cache, const int *pos,
                                       int H, int KV, int hd, int max_seq, int window, float *scratch, float *out,
                                       void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!q || !k_cache || !v_cache || !pos || !scratch || !out) return set_status(B200Q_EINVAL, "attn: null pointer");
    g_launches += 2;
    return cuda_status(launch_attn_decode(q, k_cache, v_cache, pos, H, KV, hd, max_seq, window, scratch, out,
                                          (cudaStream_t)stream),
                       "attn_decode_ex");
}

B200Q_API int b200q_argmax_dev(const float *logits, int V, int *token, int *pos, int *out_tokens, int max_tokens,
                               unsigned long long *key, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!logits || !token) return set_status(B200Q_EINVAL, "argmax: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    g_launches += key ? 2 : 1;
    return cuda_status(launch_argmax(logits, V, token, pos, out_tokens, max_tokens, key, di->sms,
                                     (cudaStream_t)stream),
                       "argmax");
}

B200Q_API size_t b200q_attn_prefill_tc_scratch_bytes(int T, int H, int KV, int hd, int max_seq)
{
    return attn_prefill_tc_scratch_bytes(T, H, KV, hd, max_seq);
}

B200Q_API int b200q_attn_prefill_tc_dev(const float *qkv, const float *k_cache, const float *v_cache, const int *pos,
                                        int T, int H, int KV, int hd, int max_seq, void *scratch,
                                        size_t scratch_bytes, void *out_bf16, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!qkv || !k_cache || !v_cache || !pos || !out_bf16 || !scratch)
        return set_status(B200Q_EINVAL, "attn_prefill_tc: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    g_launches += 2;
    return cuda_status(launch_attn_prefill_tc(qkv, k_cache, v_cache, pos, T, H, KV, hd, max_seq, scratch,
                                              scratch_bytes, static_cast<__nv_bfloat16 *>(out_bf16), di->err, di->sms,
                                              (cudaStream_t)stream),
                       "attn_prefill_tc");
}

B200Q_API int b200q_attn_prefill_dev(const float *qkv, const float *k_cache, const float *v_cache, const int *pos, int T,
                                     int H, int KV, int hd, int max_seq, void *out_bf16, void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!qkv || !k_cache || !v_cache || !pos || !out_bf16) return set_status(B200Q_EINVAL, "attn_prefill: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_attn_prefill(qkv, k_cache, v_cache, pos, T, H, KV, hd, max_seq, 0,
                                           static_cast<__nv_bfloat16 *>(out_bf16), di->err, (cudaStream_t)stream),
                       "attn_prefill");
}

B200Q_API int b200q_attn_prefill_ex_dev(const float *qkv, const float *k_cache, const float *v_cache, const int *pos,
                                        int T, int H, int KV, int hd, int max_seq, int window, void *out_bf16,
                                        void *stream)
{
    std::lock_guard<std::recursive_mutex> g(g_lock);
    if (!qkv || !k_cache || !v_cache || !pos || !out_bf16) return set_status(B200Q_EINVAL, "attn_prefill: null pointer");
    DevInfo *di = nullptr;
    if (current_device_info(&di) != B200Q_OK) return g_status;
    ++g_launches;
    return cuda_status(launch_attn_prefill(qkv, k_cache, v_cache, pos, T, H, KV, hd, max_seq, window,
                                           static_cast<__nv_bfloat16 *>(out_bf16), di->err, (cudaStream_t)stream),
                       "attn_prefill_ex");
}
