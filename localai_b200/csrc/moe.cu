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
// f32 and deterministic.  One CTA computes 64 tokens x 64 experts over a K
// range; its 256 threads are four K-slices of 64 threads, each thread holding
// 8 tokens x 8 experts (16 FMAs per 128-bit shared load), and the four slices'
// sums are added in a fixed order at the end.  For few tokens the K range is
// also split across CTAs (gridDim.z = S); those partials are written to a
// scratch array [S, T, E] and summed, in z order, by the top-k kernel.
constexpr int RT_TOK = 64, RT_EXP = 64, RT_BK = 128, RT_PAD = 4;
constexpr int RT_TILE = RT_TOK * (RT_BK + RT_PAD);   // floats per operand tile

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem), "r"(src_bytes)
                 : "memory");
}

// Double-buffered (cp.async) tiles: [buf][h | w][64 rows][RT_BK + RT_PAD].
// With ``hb`` the CTAs of the first expert tile also write bf16(h) for their
// token and K range from the staged tile (the routed rows the tensor-core
// experts gather, converted while h passes through shared memory anyway).
__global__ void __launch_bounds__(256) moe_router_kernel(const float *__restrict__ h, const float *__restrict__ wr,
                                                         const float *__restrict__ bias, float *__restrict__ out,
                                                         int T, int E, int D, int kchunk, __nv_bfloat16 *__restrict__ hb)
{
    extern __shared__ __align__(16) float rsm[];
    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * RT_TOK, e0 = blockIdx.y * RT_EXP;
    const int kbeg = blockIdx.z * kchunk, kend = min(D, kbeg + kchunk);
    const int slice = tid >> 6, lt = tid & 63;
    const int tt = lt >> 3, ee = lt & 7;              // tokens tt + 8i, experts ee + 8j
    auto load_tile = [&](int buf, int k0) {
        float *hs = rsm + buf * 2 * RT_TILE, *ws = hs + RT_TILE;
        for (int i = tid; i < RT_TOK * RT_BK / 4; i += 256) {
            const int r = i / (RT_BK / 4), c = (i % (RT_BK / 4)) * 4;
            const int t = t0 + r, e = e0 + r, kk = k0 + c;
            const bool hv = t < T && kk < kend, wv = e < E && kk < kend;
            cp_async16(hs + r * (RT_BK + RT_PAD) + c, hv ? h + (long long)t * D + kk : h, hv ? 16 : 0);
            cp_async16(ws + r * (RT_BK + RT_PAD) + c, wv ? wr + (long long)e * D + kk : wr, wv ? 16 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    if (kbeg < kend) load_tile(0, kbeg);
    int buf = 0;
    for (int k0 = kbeg; k0 < kend; k0 += RT_BK, buf ^= 1) {
        if (k0 + RT_BK < kend) {
            load_tile(buf ^ 1, k0 + RT_BK);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const float *hs = rsm + buf * 2 * RT_TILE, *ws = hs + RT_TILE;
        if (hb && blockIdx.y == 0) {
            for (int i = tid; i < RT_TOK * RT_BK / 4; i += 256) {
                const int r = i / (RT_BK / 4), c = (i % (RT_BK / 4)) * 4;
                const int t = t0 + r, kk = k0 + c;
                if (t < T && kk < kend) {
                    const float4 v = *reinterpret_cast<const float4 *>(hs + r * (RT_BK + RT_PAD) + c);
                    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
                    *reinterpret_cast<uint2 *>(hb + (long long)t * D + kk) =
                        make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
                }
            }
        }
        const int cb = slice * (RT_BK / 4);
#pragma unroll 2
        for (int c = cb; c < cb + RT_BK / 4; c += 4) {
            float4 a[8], b[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = *reinterpret_cast<const float4 *>(hs + (tt + 8 * i) * (RT_BK + RT_PAD) + c);
#pragma unroll
            for (int j = 0; j < 8; ++j) b[j] = *reinterpret_cast<const float4 *>(ws + (ee + 8 * j) * (RT_BK + RT_PAD) + c);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    acc[i][j] = fmaf(a[i].w, b[j].w, fmaf(a[i].z, b[j].z, fmaf(a[i].y, b[j].y, fmaf(a[i].x, b[j].x, acc[i][j]))));
        }
        __syncthreads();
    }
    // fixed-order reduction of the four K-slices (reuses the tile buffers)
    float *red = rsm;                                 // [3][64 tokens][64 experts]
    if (slice > 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) red[((slice - 1) * RT_TOK + tt + 8 * i) * RT_EXP + ee + 8 * j] = acc[i][j];
    }
    __syncthreads();
    if (slice == 0) {
        float *dst = out + (long long)blockIdx.z * T * E;
        const bool final = gridDim.z == 1;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int t = t0 + tt + 8 * i, e = e0 + ee + 8 * j;
                float v = acc[i][j];
#pragma unroll
                for (int s2 = 0; s2 < 3; ++s2) v += red[(s2 * RT_TOK + tt + 8 * i) * RT_EXP + ee + 8 * j];
                if (t < T && e < E) dst[(long long)t * E + e] = final ? v + (bias ? bias[e] : 0.f) : v;
            }
    }
}

// ---------------------------------------------------------------- top-k
// One warp per token; E <= 32 * EPL.
// With nsplit > 0, ``logits`` holds nsplit partial sums [nsplit, T, E] of the
// router product: they are added in split order, plus ``bias``, and the final
// logits are written to ``logits_out``.
template <int EPL>
__global__ void moe_topk_kernel(const float *__restrict__ logits, const float *__restrict__ sel_bias, int T, int E,
                                int k, int renorm, int *__restrict__ ids, float *__restrict__ wts, int nsplit,
                                const float *__restrict__ bias, float *__restrict__ logits_out)
{
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float *lr = logits + (long long)warp * E;
    float p[EPL], sel[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        if (nsplit > 0) {
            float v = 0.f;
            if (e < E) {
                for (int z = 0; z < nsplit; ++z) v += lr[(long long)z * T * E + e];
                v += bias ? bias[e] : 0.f;
                logits_out[(long long)warp * E + e] = v;
            }
            p[i] = e < E ? v : -INFINITY;
        } else {
            p[i] = e < E ? lr[e] : -INFINITY;
        }
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
        } else if (valid) {
            slot_of[i0 + item] = -1;       // a pair with a bad expert id owns no slot
        }
        __syncthreads();
        for (int i = tid; i < 8 * E; i += 256) wcnt[i] = 0;
        __syncthreads();
    }
}

// Source token of slot row ``row``, or -1 when the row must not be read: rows
// at or past ``n_valid`` (*n_valid = the dispatch's offsets[E]; slots past it
// belong to pairs with a bad expert id and were never assigned) and token ids
// outside [0, T) (recorded in the error word).
__device__ __forceinline__ int gather_token(const int *__restrict__ token_of, long long row,
                                            const int *__restrict__ n_valid, int T, int *err)
{
    if (n_valid && row >= __ldg(n_valid)) return -1;
    const int t = token_of[row];
    if (t < 0 || t >= T) {
        if ((threadIdx.x & 31) == 0) atomicExch(err, ERR_BAD_INDEX);
        return -1;
    }
    return t;
}

// out[slot, :] = h[token_of[slot], :] (f32, for the GEMV decode path); one warp per row.
__global__ void moe_gather_f32_kernel(const float *__restrict__ h, int T, const int *__restrict__ token_of,
                                      long long S, int D, float *__restrict__ out, int *err)
{
    const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= S) return;
    const int t = gather_token(token_of, row, nullptr, T, err);
    if (t < 0) return;
    const float4 *src = reinterpret_cast<const float4 *>(h + (long long)t * D);
    float4 *dst = reinterpret_cast<float4 *>(out + row * D);
    for (int c = lane; c < D / 4; c += 32) dst[c] = __ldg(src + c);
}

cudaError_t launch_moe_gather_f32(const float *h, int T, const int *token_of, int S, int D, float *out, int *err,
                                  cudaStream_t st)
{
    if (S < 1 || T < 1 || D < 4 || D % 4 || (reinterpret_cast<uintptr_t>(h) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    moe_gather_f32_kernel<<<(unsigned)(((long long)S * 32 + 255) / 256), 256, 0, st>>>(h, T, token_of, S, D, out,
                                                                                       err);
    return cudaGetLastError();
}

// out[s, :] = h[token_of[s], :] for bf16 rows (D % 8 == 0, 16-byte aligned);
// one warp per row, four 16-byte loads in flight per lane.
__global__ void moe_gather_bf16_kernel(const __nv_bfloat16 *__restrict__ h, int T, const int *__restrict__ token_of,
                                       long long S, int D, __nv_bfloat16 *__restrict__ out, int *err)
{
    const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= S) return;
    const int t = gather_token(token_of, row, nullptr, T, err);
    if (t < 0) return;
    const uint4 *src = reinterpret_cast<const uint4 *>(h + (long long)t * D);
    uint4 *dst = reinterpret_cast<uint4 *>(out + row * D);
    const int n = D / 8;
    int c = lane;
    for (; c + 96 < n; c += 128) {
        const uint4 v0 = __ldg(src + c), v1 = __ldg(src + c + 32), v2 = __ldg(src + c + 64), v3 = __ldg(src + c + 96);
        dst[c] = v0;
        dst[c + 32] = v1;
        dst[c + 64] = v2;
        dst[c + 96] = v3;
    }
    for (; c < n; c += 32) dst[c] = __ldg(src + c);
}

cudaError_t launch_moe_gather_bf16(const __nv_bfloat16 *h, int T, const int *token_of, int S, int D,
                                   __nv_bfloat16 *out, int *err, cudaStream_t st)
{
    if (S < 1 || T < 1 || D < 8 || D % 8 || (reinterpret_cast<uintptr_t>(h) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    moe_gather_bf16_kernel<<<(unsigned)(((long long)S * 32 + 255) / 256), 256, 0, st>>>(h, T, token_of, S, D, out,
                                                                                        err);
    return cudaGetLastError();
}

// The same rows written the other way round: out[slot_of[t*k + j], :] =
// h[t, :] for every token t and j < k whose pair owns a slot (slot_of >= 0).
// One warp per token reads its row once (16 loads of 16 bytes in flight per
// lane for a 4096-wide row) and stores it k times, so the source rows cross
// the memory system once instead of k times (k <= 32).  A slot at or past S
// is an error and is skipped.
__global__ void moe_scatter_bf16_kernel(const __nv_bfloat16 *__restrict__ h, int T, const int *__restrict__ slot_of,
                                        int k, long long S, int D, __nv_bfloat16 *__restrict__ out, int *err)
{
    const long long t = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (t >= T) return;
    int mine = lane < k ? __ldg(slot_of + t * k + lane) : -1;
    if (mine >= S) {
        atomicExch(err, ERR_BAD_INDEX);
        mine = -1;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(h + t * D);
    const int n = D / 8;
    for (int c0 = 0; c0 < n; c0 += 16 * 32) {
        uint4 r[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
            if (c0 + 32 * u + lane < n) r[u] = __ldg(src + c0 + 32 * u + lane);
        for (int j = 0; j < k; ++j) {
            const int slot = __shfl_sync(0xffffffffu, mine, j);
            if (slot < 0) continue;                                   // warp-uniform
            uint4 *dst = reinterpret_cast<uint4 *>(out + (long long)slot * D);
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (c0 + 32 * u + lane < n) dst[c0 + 32 * u + lane] = r[u];
        }
    }
}

cudaError_t launch_moe_scatter_bf16(const __nv_bfloat16 *h, int T, const int *slot_of, int k, int S, int D,
                                    __nv_bfloat16 *out, int *err, cudaStream_t st)
{
    if (S < 1 || T < 1 || k < 1 || k > 32 || D < 8 || D % 8 || (reinterpret_cast<uintptr_t>(h) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    moe_scatter_bf16_kernel<<<(unsigned)(((long long)T * 32 + 255) / 256), 256, 0, st>>>(h, T, slot_of, k, S, D, out,
                                                                                        err);
    return cudaGetLastError();
}

// xperm[slot, :] = bf16(h[token_of[slot], :]) for slots below offsets[E]; one warp per slot row.
__global__ void moe_gather_kernel(const float *__restrict__ h, int T, const int *__restrict__ token_of, long long S,
                                  const int *__restrict__ n_valid, int D, __nv_bfloat16 *__restrict__ xperm, int *err)
{
    const long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= S) return;
    const int t = gather_token(token_of, row, n_valid, T, err);
    if (t < 0) return;
    const float4 *src = reinterpret_cast<const float4 *>(h + (long long)t * D);
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

// bf16 rows, k <= 32: the token's slots and weights read once into shared
// memory, then each thread sums 8 consecutive values of every routed row
// (16-byte loads, the k loads of a chunk issued before their FMAs); the sum
// keeps the fixed j order, so results equal moe_combine_kernel's bit for bit.
// A slot outside [0, n_rows) adds nothing.
__global__ void __launch_bounds__(256) moe_combine_bf16x8_kernel(const __nv_bfloat16 *__restrict__ out,
                                                                 long long n_rows, const int *__restrict__ slot_of,
                                                                 const float *__restrict__ slot_w, int T, int k, int D,
                                                                 float *__restrict__ y)
{
    __shared__ long long row_s[32];
    __shared__ float w_s[32];
    const int t = blockIdx.x;
    if (t >= T) return;
    if (threadIdx.x < k) {
        const int slot = slot_of[(long long)t * k + threadIdx.x];
        const bool ok = slot >= 0 && slot < n_rows;
        row_s[threadIdx.x] = ok ? (long long)slot * (D / 8) : -1;
        w_s[threadIdx.x] = ok ? (slot_w ? __ldg(slot_w + slot) : 1.0f) : 0.f;
    }
    __syncthreads();
    const uint4 *src = reinterpret_cast<const uint4 *>(out);
    for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j0 = 0; j0 < k; j0 += 8) {
            uint4 v[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const int j = j0 + jj;
                v[jj] = (j < k && row_s[j] >= 0) ? __ldg(src + row_s[j] + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
                const int j = j0 + jj;
                if (j >= k || row_s[j] < 0) continue;
                const float wj = w_s[j];
                const uint32_t u[4] = {v[jj].x, v[jj].y, v[jj].z, v[jj].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    acc[2 * e] = fmaf(wj, __uint_as_float(u[e] << 16), acc[2 * e]);
                    acc[2 * e + 1] = fmaf(wj, __uint_as_float(u[e] & 0xffff0000u), acc[2 * e + 1]);
                }
            }
        }
        float4 *dst = reinterpret_cast<float4 *>(y + (long long)t * D) + 2 * c;
        dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// A slot outside [0, n_rows) (a pair with a bad expert id, slot -1) adds nothing.
template <typename RowT>
__global__ void moe_combine_kernel(const RowT *__restrict__ out, long long n_rows, const int *__restrict__ slot_of,
                                   const float *__restrict__ slot_w, int T, int k, int D, float *__restrict__ y)
{
    const int t = blockIdx.x;
    if (t >= T) return;
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < k; ++j) {
            const int slot = slot_of[(long long)t * k + j];
            if (slot < 0 || slot >= n_rows) continue;
            const float4 v = load4(out, (long long)slot * (D / 4) + c);
            const float wj = slot_w ? __ldg(slot_w + slot) : 1.0f;
            acc.x = fmaf(wj, v.x, acc.x); acc.y = fmaf(wj, v.y, acc.y);
            acc.z = fmaf(wj, v.z, acc.z); acc.w = fmaf(wj, v.w, acc.w);
        }
        reinterpret_cast<float4 *>(y + (long long)t * D)[c] = acc;
    }
}

// ---------------------------------------------------------------- launchers
static size_t router_smem() { return (size_t)4 * RT_TILE * sizeof(float); }

static cudaError_t router_launch(const float *h, const float *wr, const float *bias, float *out, int T, int E, int D,
                                 int nsplit, cudaStream_t st, __nv_bfloat16 *hb = nullptr)
{
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(moe_router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)router_smem());
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const int kchunk = ((D + nsplit - 1) / nsplit + RT_BK - 1) / RT_BK * RT_BK;
    dim3 grid((T + RT_TOK - 1) / RT_TOK, (E + RT_EXP - 1) / RT_EXP, nsplit);
    moe_router_kernel<<<grid, 256, router_smem(), st>>>(h, wr, bias, out, T, E, D, kchunk, hb);
    return cudaGetLastError();
}

static bool router_args_ok(const float *h, const float *wr, int T, int E, int D)
{
    return T >= 1 && E >= 1 && D >= 4 && D % 4 == 0 && !(reinterpret_cast<uintptr_t>(h) & 15) &&
           !(reinterpret_cast<uintptr_t>(wr) & 15);
}

cudaError_t launch_moe_router(const float *h, const float *wr, const float *bias, float *logits, int T, int E, int D,
                              cudaStream_t st)
{
    if (!router_args_ok(h, wr, T, E, D)) return cudaErrorInvalidValue;
    return router_launch(h, wr, bias, logits, T, E, D, 1, st);
}

template <typename... Args>
static void topk_dispatch(int E, int grid, int threads, cudaStream_t st, Args... args)
{
    if (E <= 32) moe_topk_kernel<1><<<grid, threads, 0, st>>>(args...);
    else if (E <= 64) moe_topk_kernel<2><<<grid, threads, 0, st>>>(args...);
    else if (E <= 128) moe_topk_kernel<4><<<grid, threads, 0, st>>>(args...);
    else moe_topk_kernel<8><<<grid, threads, 0, st>>>(args...);
}

cudaError_t launch_moe_topk(const float *logits, const float *sel_bias, int T, int E, int k, int renorm, int *ids,
                            float *wts, cudaStream_t st)
{
    if (T < 1 || E < 1 || E > 256 || k < 1 || k > 32 || k > E) return cudaErrorInvalidValue;
    const int threads = 256, grid = (int)(((long long)T * 32 + threads - 1) / threads);
    topk_dispatch(E, grid, threads, st, logits, sel_bias, T, E, k, renorm, ids, wts, 0, (const float *)nullptr,
                  (float *)nullptr);
    return cudaGetLastError();
}

// Number of K splits across CTAs for T tokens: enough CTAs for about two per
// SM, each with at least one K tile.
int moe_route_splits(int T, int E, int D, int num_sms)
{
    const long long ctas = (long long)((T + RT_TOK - 1) / RT_TOK) * ((E + RT_EXP - 1) / RT_EXP);
    int s = 1;
    while (s < 32 && ctas * s < 2LL * num_sms && (D / RT_BK) >= 2 * s) s *= 2;
    // one CTA per SM (the tiles take most of shared memory): among up to two
    // more doublings, the split whose last wave of CTAs is fullest (at most
    // 16 K tiles per split, the partials stay small next to h)
    auto waste = [&](int sp) {
        const long long n = ctas * sp, waves = (n + num_sms - 1) / num_sms;
        return (double)(waves * num_sms) / (double)n;
    };
    int best = s;
    for (int sp = 2 * s; sp <= 4 * s && sp <= 32 && (D / RT_BK) >= 2 * sp && ctas * sp <= 8LL * num_sms; sp *= 2)
        if (waste(sp) < waste(best) - 0.05) best = sp;
    return best;
}

size_t moe_route_workspace_bytes(int T, int E, int D, int num_sms)
{
    const int s = moe_route_splits(T, E, D, num_sms);
    return s > 1 ? (size_t)s * T * E * sizeof(float) : 0;
}

// Router + top-k in two launches; partial sums in ``ws`` when the K range is
// split across CTAs.
cudaError_t launch_moe_route(const float *h, const float *wr, const float *bias, const float *sel_bias, int T, int E,
                             int D, int k, int renorm, float *logits, int *ids, float *wts, float *ws,
                             size_t ws_bytes, int num_sms, cudaStream_t st, __nv_bfloat16 *hb)
{
    if (!router_args_ok(h, wr, T, E, D) || E > 256 || k < 1 || k > 32 || k > E) return cudaErrorInvalidValue;
    if (hb && (reinterpret_cast<uintptr_t>(hb) & 7)) return cudaErrorInvalidValue;
    int s = moe_route_splits(T, E, D, num_sms);
    if (s > 1 && (!ws || ws_bytes < (size_t)s * T * E * sizeof(float))) s = 1;
    const int threads = 256, grid = (int)(((long long)T * 32 + threads - 1) / threads);
    cudaError_t e;
    if (s == 1) {
        e = router_launch(h, wr, bias, logits, T, E, D, 1, st, hb);
        if (e != cudaSuccess) return e;
        topk_dispatch(E, grid, threads, st, (const float *)logits, sel_bias, T, E, k, renorm, ids, wts, 0,
                      (const float *)nullptr, (float *)nullptr);
    } else {
        e = router_launch(h, wr, nullptr, ws, T, E, D, s, st, hb);
        if (e != cudaSuccess) return e;
        topk_dispatch(E, grid, threads, st, (const float *)ws, sel_bias, T, E, k, renorm, ids, wts, s, bias, logits);
    }
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
    if (T < 1 || k < 1 || E < 1 || E > 4096) return cudaErrorInvalidValue;
    // the gather reads h with 16-byte loads and writes xperm with 8-byte stores
    if (xperm && (D < 4 || D % 4 || (reinterpret_cast<uintptr_t>(h) & 15) || (reinterpret_cast<uintptr_t>(xperm) & 7)))
        return cudaErrorInvalidValue;
    const int nblk = moe_num_blocks(T);
    moe_count_kernel<<<nblk, 256, E * sizeof(int), st>>>(ids, T, k, E, block_counts, err);
    moe_scan_kernel<<<1, 256, E * sizeof(int), st>>>(block_counts, nblk, E, base, offsets);
    moe_assign_kernel<<<nblk, 256, 9 * E * sizeof(int), st>>>(ids, wts, T, k, E, base, slot_of, token_of, slot_w);
    if (xperm) {
        const long long S = (long long)T * k;
        moe_gather_kernel<<<(unsigned)((S * 32 + 255) / 256), 256, 0, st>>>(h, T, token_of, S, offsets + E, D, xperm,
                                                                            err);
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
// because each call writes every count and base entry it later reads.  The
// error word (set on a bad expert id or token index) is cumulative: it is read
// and cleared by b200q_check_device_error together with the library's
// per-device error word.  Calls that overlap on the GPU (different streams, or
// different host threads without ordering) race on the array.
constexpr int NOALLOC_DISPATCH_MAX = 32768;
constexpr int NOALLOC_ERR_WORD = 2 * NOALLOC_DISPATCH_MAX;
static __device__ __align__(256) int g_noalloc_dispatch_scratch[2 * NOALLOC_DISPATCH_MAX + 64];

// Device address of the array on the current device.  Looked up on every
// call (cheap, allocates nothing), so a device reset or a reload of the
// library's module never leaves a stale address behind.
static cudaError_t noalloc_dispatch_scratch(int **ptr)
{
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_dispatch_scratch);
    if (e != cudaSuccess) return e;
    *ptr = static_cast<int *>(p);
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
    int *err = scratch + NOALLOC_ERR_WORD;
    return launch_moe_dispatch(ids, wts, T, k, E, h, D, block_counts, base, offsets, slot_of, token_of, slot_w, xperm,
                               err, st);
}

// Reads and clears the allocation-free dispatch's error word on the current
// device (synchronous; no allocation).  *code = 0 when no error was recorded.
cudaError_t noalloc_dispatch_take_error(int *code)
{
    *code = 0;
    cudaError_t e = cudaMemcpyFromSymbol(code, g_noalloc_dispatch_scratch, sizeof(int),
                                         NOALLOC_ERR_WORD * sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess || *code == 0) return e;
    const int zero = 0;
    return cudaMemcpyToSymbol(g_noalloc_dispatch_scratch, &zero, sizeof(int), NOALLOC_ERR_WORD * sizeof(int),
                              cudaMemcpyHostToDevice);
}

int noalloc_dispatch_max() { return NOALLOC_DISPATCH_MAX; }

// n_rows: rows of ``out`` (slots at or past it are skipped like unassigned ones).
cudaError_t launch_moe_combine(const void *out, bool out_bf16, long long n_rows, const int *slot_of,
                               const float *slot_w, int T, int k, int D, float *y, cudaStream_t st)
{
    if (T < 1 || k < 1 || D < 4 || D % 4 || n_rows < 1 || (reinterpret_cast<uintptr_t>(y) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & (out_bf16 ? 7 : 15)))
        return cudaErrorInvalidValue;
    if (out_bf16 && D % 8 == 0 && k <= 32 && !(reinterpret_cast<uintptr_t>(out) & 15))
        moe_combine_bf16x8_kernel<<<T, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(out), n_rows, slot_of,
                                                     slot_w, T, k, D, y);
    else if (out_bf16)
        moe_combine_kernel<__nv_bfloat16><<<T, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(out), n_rows, slot_of,
                                                             slot_w, T, k, D, y);
    else
        moe_combine_kernel<float><<<T, 256, 0, st>>>(static_cast<const float *>(out), n_rows, slot_of, slot_w, T, k,
                                                     D, y);
    return cudaGetLastError();
}

} // namespace b200q
