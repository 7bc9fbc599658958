// Mixture-of-experts routing, dispatch and combine (sm_100a).
//
// The reference MoE block (engine/zaya.py:274-307) routes one token at a time:
// router logits, softmax (f32, max-subtracted, :290), optional additive
// selection bias (:295), argmax (:296), expert FFN, scale by the unbiased
// probability (:306).  Here the same steps run batched over T tokens and
// generalised to top-k:
//   router   logits[t, e] = h[t] . Wr[e] + bias[e]          (f32, fixed order)
//   top-k    p = softmax(logits[t]); sel = p + sel_bias; k largest sel, lower
//            expert index first on ties; weight p[e] or p[e] / sum_topk p
//   dispatch stable counting sort of the (token, j) pairs by expert: slot
//            order inside an expert follows token order, so the whole layer is
//            deterministic; rows are gathered into a bf16 matrix grouped by
//            expert (the tensor-core GEMM's B operand)
//   combine  y[t] = sum_j out[slot(t, j)] for j = 0..k-1 in that order (the
//            expert outputs already carry their routing weight)
#include "common.cuh"

namespace b200q {

// ---------------------------------------------------------------- router
// f32, deterministic.  One CTA computes 16 tokens x 64 experts; its 256 threads
// form two halves that each sweep half of every 128-wide K tile (thread:
// 2 tokens x 4 experts, 128-bit shared loads along K), and the two halves'
// sums are added in a fixed order at the end.  T/16 CTAs keep the GPU busy
// even for a few thousand tokens.  Thread (tp, eq) owns tokens 2tp, 2tp+1 and
// experts eq + 16j, so the 16 lanes of a half-warp read 16 consecutive rows of
// the padded W tile (8 distinct 16-byte bank groups).
constexpr int RT_TOK = 16, RT_EXP = 64, RT_BK = 128, RT_PAD = 4;

__global__ void __launch_bounds__(256) moe_router_kernel(const float *__restrict__ h, const float *__restrict__ wr,
                                                         const float *__restrict__ bias, float *__restrict__ logits,
                                                         int T, int E, int D)
{
    __shared__ __align__(16) float hs[RT_TOK][RT_BK + RT_PAD];
    __shared__ __align__(16) float ws[RT_EXP][RT_BK + RT_PAD];
    __shared__ float part[RT_TOK][RT_EXP];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * RT_TOK, e0 = blockIdx.y * RT_EXP;
    const int half = tid >> 7, lt = tid & 127;
    const int tp = lt >> 4, eq = lt & 15;             // token pair 0..7, expert quad 0..15
    float acc[2][4] = {};
    for (int k0 = 0; k0 < D; k0 += RT_BK) {
        // h tile: 16 x 128 floats = 512 float4; W tile: 64 x 128 = 2048 float4
        for (int i = tid; i < RT_TOK * RT_BK / 4; i += 256) {
            const int r = i / (RT_BK / 4), c = (i % (RT_BK / 4)) * 4;
            const int t = t0 + r, kk = k0 + c;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < T && kk + 3 < D) v = __ldg(reinterpret_cast<const float4 *>(h + (long long)t * D + kk));
            *reinterpret_cast<float4 *>(&hs[r][c]) = v;
        }
        for (int i = tid; i < RT_EXP * RT_BK / 4; i += 256) {
            const int r = i / (RT_BK / 4), c = (i % (RT_BK / 4)) * 4;
            const int e = e0 + r, kk = k0 + c;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < E && kk + 3 < D) v = __ldg(reinterpret_cast<const float4 *>(wr + (long long)e * D + kk));
            *reinterpret_cast<float4 *>(&ws[r][c]) = v;
        }
        __syncthreads();
        const int kb = half * (RT_BK / 2);
#pragma unroll 4
        for (int c = kb; c < kb + RT_BK / 2; c += 4) {
            const float4 a0 = *reinterpret_cast<const float4 *>(&hs[2 * tp][c]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&hs[2 * tp + 1][c]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 b = *reinterpret_cast<const float4 *>(&ws[eq + 16 * j][c]);
                acc[0][j] = fmaf(a0.x, b.x, fmaf(a0.y, b.y, fmaf(a0.z, b.z, fmaf(a0.w, b.w, acc[0][j]))));
                acc[1][j] = fmaf(a1.x, b.x, fmaf(a1.y, b.y, fmaf(a1.z, b.z, fmaf(a1.w, b.w, acc[1][j]))));
            }
        }
        __syncthreads();
    }
    if (half == 1) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) part[2 * tp + i][eq + 16 * j] = acc[i][j];
    }
    __syncthreads();
    if (half == 0) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int t = t0 + 2 * tp + i, e = e0 + eq + 16 * j;
                if (t < T && e < E)
                    logits[(long long)t * E + e] = (acc[i][j] + part[2 * tp + i][eq + 16 * j]) + (bias ? bias[e] : 0.f);
            }
    }
}

// ---------------------------------------------------------------- top-k
// One warp per token; E <= 32 * EPL.
template <int EPL>
__global__ void moe_topk_kernel(const float *__restrict__ logits, const float *__restrict__ sel_bias, int T, int E,
                                int k, int renorm, int *__restrict__ ids, float *__restrict__ wts)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float *lr = logits + (long long)warp * E;
    float p[EPL], sel[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        p[i] = e < E ? lr[e] : -INFINITY;
        m = fmaxf(m, p[i]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        p[i] = e < E ? expf(p[i] - m) : 0.f;
        s += p[i];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        p[i] = p[i] / s;
        sel[i] = e < E ? (sel_bias ? p[i] + sel_bias[e] : p[i]) : -INFINITY;
    }
    float total = 0.f, chosen_p = 0.f;
    int chosen_e = -1;
    for (int j = 0; j < k; ++j) {
        float bv = -INFINITY;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const int e = lane + 32 * i;
            if (e < E && (sel[i] > bv || (sel[i] == bv && e < be))) { bv = sel[i]; be = e; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
        }
        float pv = 0.f;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
            if (lane + 32 * i == be) { pv = p[i]; sel[i] = -INFINITY; }
        pv = __shfl_sync(0xffffffffu, pv, be & 31);
        total += pv;
        if (lane == j) { chosen_e = be; chosen_p = pv; }
    }
    if (lane < k) {
        ids[(long long)warp * k + lane] = chosen_e;
        wts[(long long)warp * k + lane] = renorm ? chosen_p / total : chosen_p;
    }
}

// ---------------------------------------------------------------- dispatch
constexpr int MOE_TB = 256;       // tokens per dispatch block

__global__ void moe_count_kernel(const int *__restrict__ ids, int T, int k, int E, int *__restrict__ block_counts,
                                 int *err)
{
    extern __shared__ int cnt[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const long long i0 = (long long)blockIdx.x * MOE_TB * k;
    const long long n = min((long long)MOE_TB * k, (long long)T * k - i0);
    for (long long i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = ids[i0 + i];
        if (e < 0 || e >= E) { atomicExch(err, ERR_BAD_INDEX); continue; }
        atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) block_counts[(long long)blockIdx.x * E + e] = cnt[e];
}

// offsets[e] = rows of experts < e; base[b][e] = offsets[e] + rows of expert e in blocks < b.
__global__ void moe_scan_kernel(const int *__restrict__ block_counts, int nblk, int E, int *__restrict__ base,
                                int *__restrict__ offsets)
{
    extern __shared__ int tot[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int s = 0;
        for (int b = 0; b < nblk; ++b) s += block_counts[(long long)b * E + e];
        tot[e] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int e = 0; e < E; ++e) {
            const int c = tot[e];
            tot[e] = run;
            offsets[e] = run;
            run += c;
        }
        offsets[E] = run;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int run = tot[e];
        for (int b = 0; b < nblk; ++b) {
            base[(long long)b * E + e] = run;
            run += block_counts[(long long)b * E + e];
        }
    }
}

// Slot of every (token, j) pair, stable in (token, j) order inside each expert.
__global__ void __launch_bounds__(256) moe_assign_kernel(const int *__restrict__ ids, const float *__restrict__ wts,
                                                         int T, int k, int E, const int *__restrict__ base,
                                                         int *__restrict__ slot_of, int *__restrict__ token_of,
                                                         float *__restrict__ slot_w)
{
    extern __shared__ int sm[];
    int *running = sm;                 // [E]
    int *wcnt = sm + E;                // [8][E]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int e = tid; e < E; e += 256) running[e] = 0;
    for (int i = tid; i < 8 * E; i += 256) wcnt[i] = 0;
    __syncthreads();
    const long long i0 = (long long)blockIdx.x * MOE_TB * k;
    const int n = (int)min((long long)MOE_TB * k, (long long)T * k - i0);
    for (int r0 = 0; r0 < n; r0 += 256) {
        const int item = r0 + tid;
        const bool valid = item < n;
        int e = valid ? ids[i0 + item] : E + lane;
        if (valid && (e < 0 || e >= E)) e = E + lane;     // reported by moe_count_kernel
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const bool real = e < E;
        if (real && rank == 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        for (int ee = tid; ee < E; ee += 256) {
            int run = running[ee];
            for (int w = 0; w < 8; ++w) {
                const int c = wcnt[w * E + ee];
                wcnt[w * E + ee] = run;          // becomes the warp's exclusive prefix
                run += c;
            }
            running[ee] = run;
        }
        __syncthreads();
        if (real) {
            const int slot = base[(long long)blockIdx.x * E + e] + wcnt[warp * E + e] + rank;
            const long long gi = i0 + item;
            slot_of[gi] = slot;
            token_of[slot] = (int)(gi / k);
            slot_w[slot] = wts[gi];
        }
        __syncthreads();
        for (int i = tid; i < 8 * E; i += 256) wcnt[i] = 0;
        __syncthreads();
    }
}

// xperm[slot, :] = bf16(h[token_of[slot], :]); one warp per slot row.
__global__ void moe_gather_kernel(const float *__restrict__ h, const int *__restrict__ token_of, long long S, int D,
                                  __nv_bfloat16 *__restrict__ xperm)
{
    const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= S) return;
    const float4 *src = reinterpret_cast<const float4 *>(h + (long long)token_of[row] * D);
    uint2 *dst = reinterpret_cast<uint2 *>(xperm + row * D);
    for (int c = lane; c < D / 4; c += 32) {
        const float4 v = __ldg(src + c);
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        uint2 o;
        o.x = *reinterpret_cast<uint32_t *>(&a);
        o.y = *reinterpret_cast<uint32_t *>(&b);
        dst[c] = o;
    }
}

// y[t, :] = sum_j w_j * out[slot_of[t, j], :]   (j ascending; w_j = slot_w[slot]
// when slot_w is given, else 1 because the rows already carry their weight)
__device__ __forceinline__ float4 load4(const float *p, long long i) { return __ldg(reinterpret_cast<const float4 *>(p) + i); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16 *p, long long i)
{
    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p) + i);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
}

template <typename RowT>
__global__ void moe_combine_kernel(const RowT *__restrict__ out, const int *__restrict__ slot_of,
                                   const float *__restrict__ slot_w, int T, int k, int D, float *__restrict__ y)
{
    const int t = blockIdx.x;
    if (t >= T) return;
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; ++j) {
            const int slot = slot_of[(long long)t * k + j];
            const float4 v = load4(out, (long long)slot * (D / 4) + c);
            const float wj = slot_w ? __ldg(slot_w + slot) : 1.0f;
            acc.x = fmaf(wj, v.x, acc.x); acc.y = fmaf(wj, v.y, acc.y);
            acc.z = fmaf(wj, v.z, acc.z); acc.w = fmaf(wj, v.w, acc.w);
        }
        reinterpret_cast<float4 *>(y + (long long)t * D)[c] = acc;
    }
}

// ---------------------------------------------------------------- launchers
cudaError_t launch_moe_router(const float *h, const float *wr, const float *bias, float *logits, int T, int E, int D,
                              cudaStream_t st)
{
    if (T < 1 || E < 1 || D < 1 || D % 4 || (reinterpret_cast<uintptr_t>(h) & 15) ||
        (reinterpret_cast<uintptr_t>(wr) & 15))
        return cudaErrorInvalidValue;
    dim3 grid((T + RT_TOK - 1) / RT_TOK, (E + RT_EXP - 1) / RT_EXP);
    moe_router_kernel<<<grid, 256, 0, st>>>(h, wr, bias, logits, T, E, D);
    return cudaGetLastError();
}

cudaError_t launch_moe_topk(const float *logits, const float *sel_bias, int T, int E, int k, int renorm, int *ids,
                            float *wts, cudaStream_t st)
{
    if (T < 1 || E < 1 || E > 256 || k < 1 || k > 32 || k > E) return cudaErrorInvalidValue;
    const int threads = 256, grid = (int)(((long long)T * 32 + threads - 1) / threads);
    if (E <= 32) moe_topk_kernel<1><<<grid, threads, 0, st>>>(logits, sel_bias, T, E, k, renorm, ids, wts);
    else if (E <= 64) moe_topk_kernel<2><<<grid, threads, 0, st>>>(logits, sel_bias, T, E, k, renorm, ids, wts);
    else if (E <= 128) moe_topk_kernel<4><<<grid, threads, 0, st>>>(logits, sel_bias, T, E, k, renorm, ids, wts);
    else moe_topk_kernel<8><<<grid, threads, 0, st>>>(logits, sel_bias, T, E, k, renorm, ids, wts);
    return cudaGetLastError();
}

int moe_num_blocks(int T) { return (T + MOE_TB - 1) / MOE_TB; }

// Counting sort of the routed pairs and the bf16 gather.
//   block_counts, base: int32 [moe_num_blocks(T) * E] scratch
//   offsets: int32 [E + 1]; slot_of: int32 [T * k]; token_of: int32 [T * k];
//   slot_w: f32 [T * k]; xperm: bf16 [T * k, D] (may be null: no gather)
cudaError_t launch_moe_dispatch(const int *ids, const float *wts, int T, int k, int E, const float *h, int D,
                                int *block_counts, int *base, int *offsets, int *slot_of, int *token_of,
                                float *slot_w, __nv_bfloat16 *xperm, int *err, cudaStream_t st)
{
    if (T < 1 || k < 1 || E < 1 || E > 4096 || (xperm && D % 4)) return cudaErrorInvalidValue;
    const int nblk = moe_num_blocks(T);
    moe_count_kernel<<<nblk, 256, E * sizeof(int), st>>>(ids, T, k, E, block_counts, err);
    moe_scan_kernel<<<1, 256, E * sizeof(int), st>>>(block_counts, nblk, E, base, offsets);
    moe_assign_kernel<<<nblk, 256, 9 * E * sizeof(int), st>>>(ids, wts, T, k, E, base, slot_of, token_of, slot_w);
    if (xperm) {
        const long long S = (long long)T * k;
        moe_gather_kernel<<<(unsigned)((S * 32 + 255) / 256), 256, 0, st>>>(h, token_of, S, D, xperm);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------- allocation-free dispatch
// Callers that cannot allocate device memory -- for example a plugin running
// inside a host framework whose memory pool owns the whole device budget, or a
// latency-critical loop that must not take the implicit synchronisation of
// cudaMalloc/cudaFree -- use this variant of the dispatch.  Its scratch (the
// per-block expert counts and bases of the counting sort, and the error word)
// is a file-scope device array instead of caller or library allocations.
//
// Limit: moe_num_blocks(T) * E <= NOALLOC_DISPATCH_MAX (32768), e.g. 16384
// tokens x 512 experts or 131072 tokens x 64 experts; larger calls are
// rejected on the host.  The array occupies 256 KB + 256 B on every GPU that
// loads the library until the process exits.  Every call shares it and it
// keeps the previous call's contents; nothing in it has to start at zero,
// because each call writes every count and base entry it later reads (the
// error word is the only cumulative field, set on a bad expert id).  Calls
// that overlap on the GPU (different streams, or different host threads
// without ordering) race on the array.
constexpr int NOALLOC_DISPATCH_MAX = 32768;
static __device__ __align__(256) int g_noalloc_dispatch_scratch[2 * NOALLOC_DISPATCH_MAX + 64];

// Device address of the array, looked up once per device (with that device
// current) on the first call made on it.
cudaError_t noalloc_dispatch_scratch(int **ptr)
{
    static int *addr[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_dispatch_scratch);
        if (e != cudaSuccess) return e;
        addr[dev] = static_cast<int *>(p);
    }
    *ptr = addr[dev];
    return cudaSuccess;
}

cudaError_t launch_moe_dispatch_noalloc(const int *ids, const float *wts, int T, int k, int E, const float *h, int D,
                                        int *offsets, int *slot_of, int *token_of, float *slot_w,
                                        __nv_bfloat16 *xperm, cudaStream_t st)
{
    if (T < 1 || E < 1 || (long long)moe_num_blocks(T) * E > NOALLOC_DISPATCH_MAX) return cudaErrorInvalidValue;
    int *scratch = nullptr;
    cudaError_t e = noalloc_dispatch_scratch(&scratch);
    if (e != cudaSuccess) return e;
    int *block_counts = scratch, *base = scratch + NOALLOC_DISPATCH_MAX;
    int *err = scratch + 2 * NOALLOC_DISPATCH_MAX;
    return launch_moe_dispatch(ids, wts, T, k, E, h, D, block_counts, base, offsets, slot_of, token_of, slot_w, xperm,
                               err, st);
}

int noalloc_dispatch_max() { return NOALLOC_DISPATCH_MAX; }

cudaError_t launch_moe_combine(const void *out, bool out_bf16, const int *slot_of, const float *slot_w, int T, int k,
                               int D, float *y, cudaStream_t st)
{
    if (T < 1 || k < 1 || D % 4) return cudaErrorInvalidValue;
    if (out_bf16)
        moe_combine_kernel<__nv_bfloat16><<<T, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(out), slot_of, slot_w,
                                                             T, k, D, y);
    else
        moe_combine_kernel<float><<<T, 256, 0, st>>>(static_cast<const float *>(out), slot_of, slot_w, T, k, D, y);
    return cudaGetLastError();
}

} // namespace b200q
