// One decode step of the reference's Llama decoder around the quantised
// GEMVs (engine/model.py:174-240, LlamaModel.forward, arch 'llama'):
//
//   x = emb[token]
//   per layer:  h = rmsnorm(x) * attn_norm
//               q, k, v = Wq h, Wk h, Wv h          (one GEMV over [Wq; Wk; Wv])
//               q, k = rope(q, k, position)          adjacent pairs, rope.freq_base
//               cache[position] = k, v
//               att = softmax(q k^T / sqrt(hd)) v    grouped heads (GQA)
//               x = x + Wo att;  h = rmsnorm(x) * ffn_norm
//               x = x + Wdown (silu(Wgate h) * Wup h)
//   logits = Wout (rmsnorm(x) * output_norm);  token = argmax(logits)
//
// Every kernel here reads the position and the token from device memory, so
// one step can be captured once in a CUDA graph and replayed per token with no
// host synchronisation.  Attention splits the cached positions into chunks of
// ATT_CHUNK (one CTA per KV head and chunk, partial max / sum / weighted V),
// then combines the chunks in a fixed order.
#include "common.cuh"
#include <algorithm>

namespace b200q {

constexpr int ATT_CHUNK = 64;

// x += delta (when given); h = x / sqrt(mean(x^2) + eps) * w  (engine/model.py:82).
// One CTA of 512 threads per row; every thread loads its (up to 8) float4
// groups of x and delta before anything is stored, so the row costs one
// memory round trip; the sum of squares is reduced in a fixed order.
constexpr int NORM_THREADS = 512, NORM_VEC = 8;
__global__ void __launch_bounds__(NORM_THREADS) add_rmsnorm_kernel(float *__restrict__ x, const float *__restrict__ delta,
                                                                   const float *__restrict__ w, int D, float eps,
                                                                   float *__restrict__ h, __nv_bfloat16 *__restrict__ hb)
{
    __shared__ float red[NORM_THREADS / 32];
    pdl_enter();
    const long long t = blockIdx.x;
    float4 *xr = reinterpret_cast<float4 *>(x + t * D);
    const float4 *dr = delta ? reinterpret_cast<const float4 *>(delta + t * D) : nullptr;
    const int n4 = D / 4;
    float4 v[NORM_VEC];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NORM_VEC; ++k) {
        const int i = threadIdx.x + k * NORM_THREADS;
        v[k] = i < n4 ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (dr) {
#pragma unroll
        for (int k = 0; k < NORM_VEC; ++k) {
            const int i = threadIdx.x + k * NORM_THREADS;
            if (i < n4) {
                const float4 d = dr[i];
                v[k].x += d.x; v[k].y += d.y; v[k].z += d.z; v[k].w += d.w;
            }
        }
    }
    const float4 *wr = reinterpret_cast<const float4 *>(w);
    float4 wv[NORM_VEC];                       // norm weights: loaded before the reduction
#pragma unroll
    for (int k = 0; k < NORM_VEC; ++k) {
        const int i = threadIdx.x + k * NORM_THREADS;
        wv[k] = i < n4 ? wr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < NORM_VEC; ++k)
        ss = fmaf(v[k].w, v[k].w, fmaf(v[k].z, v[k].z, fmaf(v[k].y, v[k].y, fmaf(v[k].x, v[k].x, ss))));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < NORM_THREADS / 32; ++i) tot += red[i];
    const float inv = 1.0f / sqrtf(tot / (float)D + eps);
#pragma unroll
    for (int k = 0; k < NORM_VEC; ++k) {
        const int i = threadIdx.x + k * NORM_THREADS;
        if (i < n4) {
            if (dr) xr[i] = v[k];
            const float4 g = wv[k];
            const float4 o = make_float4(v[k].x * inv * g.x, v[k].y * inv * g.y, v[k].z * inv * g.z, v[k].w * inv * g.w);
            if (h) reinterpret_cast<float4 *>(h + t * D)[i] = o;
            if (hb) {
                __nv_bfloat162 a = __floats2bfloat162_rn(o.x, o.y), b = __floats2bfloat162_rn(o.z, o.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t *>(&a);
                u.y = *reinterpret_cast<uint32_t *>(&b);
                reinterpret_cast<uint2 *>(hb + t * D)[i] = u;
            }
        }
    }
}

// qkv = [q (H*hd) | k (KV*hd) | v (KV*hd)]: rotate q and k in place over the
// first ``rotary`` dims (adjacent pairs, engine/model.py:205-217):
// inv_j = 1 / base^(j / half) (or inv_freq[j] when a table is given),
// angle = pos * inv_j; and store the rotated k
// and v of every row into the caches (layout [max_seq][KV][hd], as the
// reference's KVCache).  Rows t of qkv (row stride (H + 2 KV) * hd) are
// positions *pos_p + t.  Work items of one row: H*half q pairs, KV*half k
// pairs (rotated, then stored), KV*(hd - rotary) unrotated k values and KV*hd
// v values (both only stored).
__global__ void rope_kv_kernel(float *__restrict__ qkv, int T, int H, int KV, int hd, int rotary, float base,
                               const float *__restrict__ inv_freq, int neox, const int *__restrict__ pos_p,
                               float *__restrict__ kc, float *__restrict__ vc, int max_seq, int *err)
{
    pdl_enter();
    const int pos0 = *pos_p;
    if (pos0 < 0 || pos0 + T > max_seq) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ERR_BAD_INDEX);
        return;
    }
    const int half = rotary / 2;
    const int nq = H * half, nk = KV * half, nkr = KV * (hd - rotary), nv = KV * hd;
    const long long per_row = (long long)nq + nk + nkr + nv;
    const long long row = (long long)(H + 2 * KV) * hd;
    const int n = KV * hd;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)T * per_row;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / per_row);
        int r = (int)(i % per_row);
        float *qr = qkv + t * row;
        float *kcr = kc + (long long)(pos0 + t) * n, *vcr = vc + (long long)(pos0 + t) * n;
        if (r < nq + nk) {                               // a rotated pair of q or k
            const bool is_k = r >= nq;
            if (is_k) r -= nq;
            const int hh = r / half, j = r % half;
            // a given frequency table (RoPE scaling: llama3 interpolation, linear) or base^(-j/half)
            const float inv = inv_freq ? __ldg(inv_freq + j) : 1.0f / powf(base, (float)j / (float)half);
            const float ang = (float)(pos0 + t) * inv;
            const float c = cosf(ang), s = sinf(ang);
            // pair j: dims (2j, 2j+1) (llama) or (j, j + half) (NeoX split halves, qwen2/qwen3)
            const int de = neox ? j : 2 * j, dodd = neox ? j + half : 2 * j + 1;
            const long long hb = (long long)((is_k ? H : 0) + hh) * hd;
            const float e = qr[hb + de], o = qr[hb + dodd];
            const float e2 = e * c - o * s, o2 = e * s + o * c;
            qr[hb + de] = e2;
            qr[hb + dodd] = o2;
            if (is_k) {
                kcr[hh * hd + de] = e2;
                kcr[hh * hd + dodd] = o2;
            }
        } else if (r < nq + nk + nkr) {                  // k beyond the rotary dims
            r -= nq + nk;
            const int hh = r / (hd - rotary), d = rotary + r % (hd - rotary);
            kcr[hh * hd + d] = qr[(long long)(H + hh) * hd + d];
        } else {                                         // v
            r -= nq + nk + nkr;
            vcr[r] = qr[(long long)(H + KV) * hd + r];
        }
    }
}

// One CTA per (KV head g, chunk c of ATT_CHUNK positions), 256 threads (8
// warps).  The G = H / KV query rows of the group, the chunk's K rows and V
// rows are staged densely in shared memory with 16-byte cp.async (all in
// flight at once).  Scores: warp w takes positions w, w + 8, ...; lane i holds
// dims 4i .. 4i+3 of the G query rows in registers, reads the same dims of the
// K row (one 128-bit shared load, no bank conflicts) and the G partial dots
// are summed across the warp with shuffles.  Warp j < G then does the softmax
// statistics of head j.  P V: warp w accumulates positions w, w + 8, ... for
// dims 4i .. 4i+3 of every head; the eight per-warp partials (stored where
// the K rows were) are added in warp order.  Writes per query head the
// chunk's max, sum of exp and exp-weighted V.  Needs hd % 4 == 0, hd <= 128,
// G <= 8.
constexpr int ATT_THREADS = 256, ATT_WARPS = ATT_THREADS / 32, ATT_MAXG = 8;

__device__ __forceinline__ void cp_async16_cg(void *smem, const void *gmem)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)), "l"(gmem)
                 : "memory");
}

__global__ void __launch_bounds__(ATT_THREADS) attn_chunk_kernel(const float *__restrict__ q, const float *__restrict__ kc,
                                                                 const float *__restrict__ vc,
                                                                 const int *__restrict__ pos_p, int H, int KV, int hd,
                                                                 int max_seq, int window, float *__restrict__ part)
{
    extern __shared__ __align__(16) float asm_[];
    pdl_enter();
    const int G = H / KV, g = blockIdx.x, c = blockIdx.y;
    const int L = min(*pos_p + 1, max_seq);
    // sliding window (engine/model.py:222): only the last ``window`` positions
    const int l0 = max(c * ATT_CHUNK, window > 0 ? L - window : 0), l1 = min(L, c * ATT_CHUNK + ATT_CHUNK);
    const int nch = gridDim.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd4 = hd >> 2;
    float *qs = asm_;                          // [G][hd]
    float *ks = qs + G * hd;                   // [ATT_CHUNK][hd]; later [ATT_WARPS][G][hd] partials of P V
    float *vs = ks + ATT_CHUNK * hd;           // [ATT_CHUNK][hd]
    float *sc = vs + ATT_CHUNK * hd;           // [G][ATT_CHUNK]
    float *stat = sc + G * ATT_CHUNK;          // [G][2]: max, sum
    // part layout: [H][nch][hd + 2]: acc[hd], max, sum
    if (l1 <= l0) {                            // chunk past the current position
        for (int i = tid; i < G * (hd + 2); i += blockDim.x) {
            const int j = i / (hd + 2), d = i % (hd + 2);
            part[((long long)(g * G + j) * nch + c) * (hd + 2) + d] = d == hd ? -INFINITY : 0.f;
        }
        return;
    }
    const int n = l1 - l0;
    for (int i = tid; i < G * hd4; i += ATT_THREADS) cp_async16_cg(qs + 4 * i, q + (long long)g * G * hd + 4 * i);
    for (int i = tid; i < n * hd4; i += ATT_THREADS) {
        const int l = i / hd4, d4 = i - l * hd4;
        const long long src = ((long long)(l0 + l) * KV + g) * hd + 4 * d4;
        cp_async16_cg(ks + l * hd + 4 * d4, kc + src);
        cp_async16_cg(vs + l * hd + 4 * d4, vc + src);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();

    const bool lv = lane < hd4;                // this lane's dims exist
    float4 qr[ATT_MAXG];
#pragma unroll
    for (int j = 0; j < ATT_MAXG; ++j)
        qr[j] = (j < G && lv) ? reinterpret_cast<const float4 *>(qs)[j * hd4 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float rs = sqrtf((float)hd);
    for (int l = warp; l < ATT_CHUNK; l += ATT_WARPS) {
        const float4 kv = (l < n && lv) ? reinterpret_cast<const float4 *>(ks)[l * hd4 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
        float s[ATT_MAXG];
#pragma unroll
        for (int j = 0; j < ATT_MAXG; ++j)
            s[j] = fmaf(qr[j].w, kv.w, fmaf(qr[j].z, kv.z, fmaf(qr[j].y, kv.y, qr[j].x * kv.x)));
#pragma unroll
        for (int j = 0; j < ATT_MAXG; ++j) {
            if (j < G) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s[j] += __shfl_xor_sync(0xffffffffu, s[j], o);
                if (lane == 0) sc[j * ATT_CHUNK + l] = l < n ? s[j] / rs : -INFINITY;
            }
        }
    }
    __syncthreads();
    for (int j = warp; j < G; j += ATT_WARPS) {
        float m = -INFINITY;
        for (int l = lane; l < ATT_CHUNK; l += 32) m = fmaxf(m, sc[j * ATT_CHUNK + l]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float sum = 0.f;
        for (int l = lane; l < ATT_CHUNK; l += 32) {
            const float e = l < n ? expf(sc[j * ATT_CHUNK + l] - m) : 0.f;
            sc[j * ATT_CHUNK + l] = e;
            sum += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[2 * j] = m;
            stat[2 * j + 1] = sum;
        }
    }
    __syncthreads();
    float4 acc[ATT_MAXG];
#pragma unroll
    for (int j = 0; j < ATT_MAXG; ++j) acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int l = warp; l < n; l += ATT_WARPS) {
        const float4 vv = lv ? reinterpret_cast<const float4 *>(vs)[l * hd4 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < ATT_MAXG; ++j) {
            if (j < G) {
                const float p = sc[j * ATT_CHUNK + l];
                acc[j].x = fmaf(p, vv.x, acc[j].x);
                acc[j].y = fmaf(p, vv.y, acc[j].y);
                acc[j].z = fmaf(p, vv.z, acc[j].z);
                acc[j].w = fmaf(p, vv.w, acc[j].w);
            }
        }
    }
    // the K rows are no longer read (scores are done): per-warp partials go there
    float *red = ks;
    if (lv) {
#pragma unroll
        for (int j = 0; j < ATT_MAXG; ++j)
            if (j < G) reinterpret_cast<float4 *>(red)[(warp * G + j) * hd4 + lane] = acc[j];
    }
    __syncthreads();
    for (int i = tid; i < G * hd; i += ATT_THREADS) {
        const int j = i / hd, d = i - j * hd;
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; ++w) a += red[(w * G + j) * hd + d];
        float *pp = part + ((long long)(g * G + j) * nch + c) * (hd + 2);
        pp[d] = a;
        if (d == 0) {
            pp[hd] = stat[2 * j];
            pp[hd + 1] = stat[2 * j + 1];
        }
    }
}

// Causal prefill attention (engine/model.py:130-160, forward_sequence): query
// row t (position *pos_p + t, rotated q in qkv row t) attends to cache
// positions 0 .. *pos_p + t.  CTA = (query head h, tile of PF_Q = 64 query
// rows), 256 threads as a 16 x 16 grid (ty, tx).  Per tile of PF_K = 64 key
// positions (K and V rows staged with 16-byte cp.async, the next tile's K
// loading during P V and its V during the next scores):
//   scores  thread (ty, tx) computes rows 4ty .. 4ty+3 x keys tx + 16j (j < 4)
//           from 128-bit shared loads (8 FMAs per load; keys interleaved by
//           16 so that the K reads of a quarter warp hit distinct banks);
//   softmax online per row (running max and sum), the 16 threads of a row
//           combine with shuffles; probabilities go to shared memory;
//   P V     thread (ty, tx) accumulates rows 4ty .. 4ty+3 x dims 64c + 4tx ..
//           64c + 4tx + 3 (c < hd / 64).
// f32 throughout; output bf16 for the O GEMM.  Needs hd = 64 or 128.
constexpr int PF_Q = 64, PF_K = 64, PF_THREADS = 256;

__global__ void __launch_bounds__(PF_THREADS) attn_prefill_kernel(const float *__restrict__ qkv,
                                                                  const float *__restrict__ kc,
                                                                  const float *__restrict__ vc,
                                                                  const int *__restrict__ pos_p, int T, int H, int KV,
                                                                  int hd, int max_seq, int window,
                                                                  __nv_bfloat16 *__restrict__ out, int *err)
{
    extern __shared__ __align__(16) float pf[];
    pdl_enter();
    const int h = blockIdx.x, t0 = blockIdx.y * PF_Q;
    if (t0 >= T) return;
    const int g = h / (H / KV);
    const int p0 = *pos_p;
    if (p0 < 0 || p0 + T > max_seq) {          // positions outside the cache: write nothing, report
        if (threadIdx.x == 0) atomicExch(err, ERR_BAD_INDEX);
        return;
    }
    const int nq = min(PF_Q, T - t0);
    const int st = hd + 4, pst = PF_K + 4, hd4 = hd >> 2, nc = hd >> 6;
    float *qs = pf;                    // [PF_Q][hd + 4]
    float *ks = qs + PF_Q * st;        // [PF_K][hd + 4]
    float *vs = ks + PF_K * st;        // [PF_K][hd + 4]
    float *ps = vs + PF_K * st;        // [PF_Q][PF_K + 4]
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const long long R = (long long)(H + 2 * KV) * hd;
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = tid; i < PF_Q * hd4; i += PF_THREADS) {
        const int rr = i / hd4, d4 = i - rr * hd4;
        float *dst = qs + rr * st + 4 * d4;
        if (rr < nq) cp_async16_cg(dst, qkv + (t0 + rr) * R + (long long)h * hd + 4 * d4);
        else *reinterpret_cast<float4 *>(dst) = zero4;
    }
    const int kmax = p0 + t0 + nq - 1;              // last key position any row of the tile sees
    // rows [k0, k0 + nk) of the cache into dst; rows nk .. PF_K-1 zero
    auto load_rows = [&](float *dst, const float *cache, int k0) {
        const int nk = min(PF_K, kmax + 1 - k0);
        for (int i = tid; i < PF_K * hd4; i += PF_THREADS) {
            const int jj = i / hd4, d4 = i - jj * hd4;
            float *d = dst + jj * st + 4 * d4;
            if (jj < nk) cp_async16_cg(d, cache + ((long long)(k0 + jj) * KV + g) * hd + 4 * d4);
            else *reinterpret_cast<float4 *>(d) = zero4;
        }
    };
    // sliding window (engine/model.py:222): row r sees keys (p0 + t0 + r - window, p0 + t0 + r];
    // key tiles before the first row's window are skipped
    const int kfirst = window > 0 ? max(0, p0 + t0 - window + 1) / PF_K * PF_K : 0;
    load_rows(ks, kc, kfirst);
    load_rows(vs, vc, kfirst);

    float m[4], l[4], acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) acc[i][d] = 0.f;
    }
    const float rs = sqrtf((float)hd);
    for (int k0 = kfirst; k0 <= kmax; k0 += PF_K) {
        const int nk = min(PF_K, kmax + 1 - k0);
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();                                  // this tile's K and V (and q) are in place
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) sc[i][jj] = 0.f;
        for (int e = 0; e < hd; e += 4) {
            float4 qv[4], kv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4 *>(qs + (4 * ty + i) * st + e);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) kv[jj] = *reinterpret_cast<const float4 *>(ks + (tx + 16 * jj) * st + e);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj)
                    sc[i][jj] = fmaf(qv[i].w, kv[jj].w,
                                     fmaf(qv[i].z, kv[jj].z, fmaf(qv[i].y, kv[jj].y, fmaf(qv[i].x, kv[jj].x, sc[i][jj]))));
        }
        float scale[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = 4 * ty + i;
            float tmax = -INFINITY;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int key = tx + 16 * jj;
                const bool ok = row < nq && key < nk && k0 + key <= p0 + t0 + row &&
                                (window <= 0 || k0 + key > p0 + t0 + row - window);
                sc[i][jj] = ok ? sc[i][jj] / rs : -INFINITY;
                tmax = fmaxf(tmax, sc[i][jj]);
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
            const float mn = fmaxf(m[i], tmax);
            scale[i] = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
            float psum = 0.f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const float p = (sc[i][jj] == -INFINITY) ? 0.f : expf(sc[i][jj] - mn);
                ps[row * pst + tx + 16 * jj] = p;
                psum += p;
            }
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
            l[i] = l[i] * scale[i] + psum;
            m[i] = mn;
#pragma unroll
            for (int d = 0; d < 8; ++d) acc[i][d] *= scale[i];
        }
        __syncthreads();                                  // probabilities complete; K no longer read
        if (k0 + PF_K <= kmax) {
            load_rows(ks, kc, k0 + PF_K);                 // next K lands during P V
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        for (int kk = 0; kk < PF_K; kk += 4) {
            float4 pv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pv[i] = *reinterpret_cast<const float4 *>(ps + (4 * ty + i) * pst + kk);
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    if (c < nc) {
                        const float4 vv = *reinterpret_cast<const float4 *>(vs + (kk + q4) * st + 64 * c + 4 * tx);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float p = q4 == 0 ? pv[i].x : q4 == 1 ? pv[i].y : q4 == 2 ? pv[i].z : pv[i].w;
                            acc[i][4 * c] = fmaf(p, vv.x, acc[i][4 * c]);
                            acc[i][4 * c + 1] = fmaf(p, vv.y, acc[i][4 * c + 1]);
                            acc[i][4 * c + 2] = fmaf(p, vv.z, acc[i][4 * c + 2]);
                            acc[i][4 * c + 3] = fmaf(p, vv.w, acc[i][4 * c + 3]);
                        }
                    }
                }
            }
        }
        __syncthreads();                                  // V and the probabilities no longer read
        if (k0 + PF_K <= kmax) {
            load_rows(vs, vc, k0 + PF_K);                 // next V lands during the next scores
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = 4 * ty + i;
        if (row < nq) {
            const float inv = 1.0f / l[i];
            __nv_bfloat16 *o = out + (long long)(t0 + row) * H * hd + (long long)h * hd;
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                if (c < nc) {
                    __nv_bfloat162 a = __floats2bfloat162_rn(acc[i][4 * c] * inv, acc[i][4 * c + 1] * inv);
                    __nv_bfloat162 b = __floats2bfloat162_rn(acc[i][4 * c + 2] * inv, acc[i][4 * c + 3] * inv);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t *>(&a);
                    u.y = *reinterpret_cast<uint32_t *>(&b);
                    *reinterpret_cast<uint2 *>(o + 64 * c + 4 * tx) = u;
                }
            }
        }
    }
}

cudaError_t launch_attn_prefill(const float *qkv, const float *kc, const float *vc, const int *pos, int T, int H,
                                int KV, int hd, int max_seq, int window, __nv_bfloat16 *out, int *err, cudaStream_t st)
{
    if (T < 1 || H < 1 || KV < 1 || H % KV || (hd != 64 && hd != 128) || max_seq < 1 || window < 0 ||
        (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(kc) & 15) ||
        (reinterpret_cast<uintptr_t>(vc) & 15) || (reinterpret_cast<uintptr_t>(out) & 7))
        return cudaErrorInvalidValue;
    const size_t smem = (size_t)((PF_Q + 2 * PF_K) * (hd + 4) + PF_Q * (PF_K + 4)) * sizeof(float);
    static size_t attr = 0;
    if (smem > attr) {
        cudaError_t e = cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr = smem;
    }
    return launch_pdl(attn_prefill_kernel, dim3(H, (T + PF_Q - 1) / PF_Q), dim3(PF_THREADS), smem, st, qkv, kc, vc, pos,
                      T, H, KV, hd, max_seq, window, out, err);
}

// out[h][d] = sum_c exp(m_c - M) acc_c[d] / sum_c exp(m_c - M) s_c, chunks in
// order.  One CTA per query head: the chunk weights exp(m_c - M) / S are
// computed once into shared memory (chunks past the position have
// m_c = -inf, weight 0), then thread d sums its column over the chunks.
constexpr int COMB_MAX_CHUNKS = 2048;
__global__ void attn_combine_kernel(const float *__restrict__ part, int nch, int hd, float *__restrict__ out)
{
    __shared__ float wsh[COMB_MAX_CHUNKS];
    __shared__ float red[32];
    pdl_enter();
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const float *ph = part + (long long)h * nch * (hd + 2);
    float mloc = -INFINITY;
    for (int c = tid; c < nch; c += blockDim.x) {
        const float mc = ph[c * (hd + 2) + hd];
        wsh[c] = mc;
        mloc = fmaxf(mloc, mc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
    if (lane == 0) red[warp] = mloc;
    __syncthreads();
    float M = -INFINITY;
    for (int i = 0; i < nw; ++i) M = fmaxf(M, red[i]);
    __syncthreads();                           // red is reused below
    float sloc = 0.f;
    for (int c = tid; c < nch; c += blockDim.x) {
        const float mc = wsh[c];
        const float e = mc == -INFINITY ? 0.f : expf(mc - M);
        wsh[c] = e;
        sloc += e * ph[c * (hd + 2) + hd + 1];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sloc += __shfl_xor_sync(0xffffffffu, sloc, o);
    if (lane == 0) red[warp] = sloc;
    __syncthreads();
    float S = 0.f;
    for (int i = 0; i < nw; ++i) S += red[i];
    for (int d = tid; d < hd; d += blockDim.x) {
        float a = 0.f;
        for (int c = 0; c < nch; ++c) a = fmaf(wsh[c], ph[c * (hd + 2) + d], a);
        out[(long long)h * hd + d] = a / S;
    }
}

// token = argmax(logits) (first index on ties, as np.argmax); the token is
// also stored at out_tokens[pos] and pos advances by one (the step's end).
__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ logits, int V, int *__restrict__ token,
                                                      int *__restrict__ pos_p, int *__restrict__ out_tokens,
                                                      int max_tokens)
{
    __shared__ float bv[1024];
    __shared__ int bi[1024];
    pdl_enter();
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = logits[i];
        if (v > best || (v == best && i < idx)) { best = v; idx = i; }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if ((int)threadIdx.x < o) {
            const float v = bv[threadIdx.x + o];
            const int i = bi[threadIdx.x + o];
            if (v > bv[threadIdx.x] || (v == bv[threadIdx.x] && i < bi[threadIdx.x])) {
                bv[threadIdx.x] = v;
                bi[threadIdx.x] = i;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int t = bi[0] == 0x7fffffff ? 0 : bi[0];
        *token = t;
        if (pos_p) {
            const int p = *pos_p;
            if (out_tokens && p >= 0 && p < max_tokens) out_tokens[p] = t;
            *pos_p = p + 1;
        }
    }
}

cudaError_t launch_add_rmsnorm(float *x, const float *delta, const float *w, int T, int D, float eps, float *h,
                               __nv_bfloat16 *hb, cudaStream_t st)
{
    if (T < 1 || D < 4 || D % 4 || D > 4 * NORM_THREADS * NORM_VEC || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(h) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
        (reinterpret_cast<uintptr_t>(hb) & 7) || (!h && !hb) || (delta && (reinterpret_cast<uintptr_t>(delta) & 15)))
        return cudaErrorInvalidValue;
    return launch_pdl(add_rmsnorm_kernel, dim3(T), dim3(NORM_THREADS), 0, st, x, delta, w, D, eps, h, hb);
}

// Before RoPE, per row t < T of qkv = [q H*hd | k KV*hd | v KV*hd]: add the
// projection bias (when given: [(H + 2 KV) * hd], engine/model.py:73-79, the
// biased Q/K/V of Qwen2), then RMS-normalise every q head and every k head
// over its hd values with the per-head weights q_norm / k_norm (when given:
// [hd], Qwen3, engine/model.py:188-192: x / sqrt(mean(x^2) + eps) * w).  One
// warp per (row, head); hd <= 256, a multiple of 32.
__global__ void qkv_bias_norm_kernel(float *__restrict__ qkv, int T, int H, int KV, int hd,
                                     const float *__restrict__ bias, const float *__restrict__ qn,
                                     const float *__restrict__ kn, float eps)
{
    pdl_enter();
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int nh = H + 2 * KV;
    if (wid >= (long long)T * nh) return;
    const int t = (int)(wid / nh), hh = (int)(wid % nh);
    float *a = qkv + ((long long)t * nh + hh) * hd;
    const float *b = bias ? bias + (long long)hh * hd : nullptr;
    const float *g = hh < H ? qn : hh < H + KV ? kn : nullptr;
    const int per = hd / 32;
    float v[8];
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u)
        if (u < per) {
            v[u] = a[lane + 32 * u] + (b ? __ldg(b + lane + 32 * u) : 0.f);
            ss += v[u] * v[u];
        }
    if (g) {
#pragma unroll
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = 1.0f / sqrtf(ss / (float)hd + eps);
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (u < per) v[u] = v[u] * r * __ldg(g + lane + 32 * u);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
        if (u < per) a[lane + 32 * u] = v[u];
}

cudaError_t launch_qkv_bias_norm(float *qkv, int T, int H, int KV, int hd, const float *bias, const float *qn,
                                 const float *kn, float eps, cudaStream_t st)
{
    if (T < 1 || H < 1 || KV < 1 || hd < 32 || hd > 256 || hd % 32) return cudaErrorInvalidValue;
    const long long warps = (long long)T * (H + 2 * KV);
    return launch_pdl(qkv_bias_norm_kernel, dim3((unsigned)((warps * 32 + 255) / 256)), dim3(256), 0, st, qkv, T, H,
                      KV, hd, bias, qn, kn, eps);
}

cudaError_t launch_rope_kv(float *qkv, int T, int H, int KV, int hd, int rotary, float base, const float *inv_freq,
                           int neox, const int *pos, float *kc, float *vc, int max_seq, int *err, int num_sms,
                           cudaStream_t st)
{
    if (T < 1 || H < 1 || KV < 1 || H % KV || hd < 2 || rotary < 0 || rotary > hd || rotary % 2 || max_seq < 1)
        return cudaErrorInvalidValue;
    const long long items = (long long)T * ((long long)(H + KV) * (rotary / 2) + (long long)KV * (hd - rotary) +
                                            (long long)KV * hd);
    const long long g = std::min(8LL * num_sms, (items + 255) / 256);
    return launch_pdl(rope_kv_kernel, dim3((unsigned)g), dim3(256), 0, st, qkv, T, H, KV, hd, rotary, base, inv_freq,
                      neox ? 1 : 0, pos, kc, vc, max_seq, err);
}

size_t attn_scratch_floats(int H, int hd, int max_seq)
{
    const int nch = (max_seq + ATT_CHUNK - 1) / ATT_CHUNK;
    return (size_t)H * nch * (hd + 2);
}

cudaError_t launch_attn_decode(const float *q, const float *kc, const float *vc, const int *pos, int H, int KV, int hd,
                               int max_seq, int window, float *part, float *out, cudaStream_t st)
{
    if (H < 1 || KV < 1 || H % KV || hd < 4 || hd > 128 || hd % 4 || H / KV > ATT_MAXG || max_seq < 1 || window < 0 ||
        (reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(kc) & 15) ||
        (reinterpret_cast<uintptr_t>(vc) & 15))
        return cudaErrorInvalidValue;
    const int G = H / KV, nch = (max_seq + ATT_CHUNK - 1) / ATT_CHUNK;
    const size_t smem = (size_t)(G * hd + 2 * ATT_CHUNK * hd + G * ATT_CHUNK + 2 * G) * sizeof(float);
    if (smem > 200 * 1024 || nch > COMB_MAX_CHUNKS) return cudaErrorInvalidValue;
    static size_t attr = 0;
    if (smem > attr) {
        cudaError_t e = cudaFuncSetAttribute(attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr = smem;
    }
    cudaError_t e = launch_pdl(attn_chunk_kernel, dim3(KV, nch), dim3(ATT_THREADS), smem, st, q, kc, vc, pos, H, KV, hd,
                               max_seq, window, part);
    if (e != cudaSuccess) return e;
    return launch_pdl(attn_combine_kernel, dim3(H), dim3(128), 0, st, part, nch, hd, out);
}

// Grid-wide argmax: every CTA reduces a slice, then one 64-bit atomicMax of
// the key (order-preserving bits of the value << 32 | ~index), so the largest
// value wins and, among equal values, the lowest index (np.argmax).  The
// finishing thread decodes the token, records it, advances pos and clears the
// key for the next step.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i)
{
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)o << 32) | (0xFFFFFFFFu - (uint32_t)i);
}

__global__ void __launch_bounds__(256) argmax_part_kernel(const float *__restrict__ logits, int V,
                                                          unsigned long long *key)
{
    __shared__ unsigned long long red[8];
    pdl_enter();
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        const unsigned long long k = argmax_key(logits[i], i);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < 8; ++i) best = red[i] > best ? red[i] : best;
        atomicMax(key, best);
    }
}

__global__ void argmax_finish_kernel(unsigned long long *key, int *token, int *pos_p, int *out_tokens, int max_tokens)
{
    pdl_enter();
    const unsigned long long k = *key;
    const int t = k ? (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
    *token = t;
    if (pos_p) {
        const int p = *pos_p;
        if (out_tokens && p >= 0 && p < max_tokens) out_tokens[p] = t;
        *pos_p = p + 1;
    }
    *key = 0ull;
}

cudaError_t launch_argmax(const float *logits, int V, int *token, int *pos, int *out_tokens, int max_tokens,
                          unsigned long long *key, int num_sms, cudaStream_t st)
{
    if (V < 1) return cudaErrorInvalidValue;
    if (!key) {
        return launch_pdl(argmax_kernel, dim3(1), dim3(1024), 0, st, logits, V, token, pos, out_tokens, max_tokens);
    }
    int grid = (V + 255) / 256;
    if (grid > num_sms) grid = num_sms;
    cudaError_t e = launch_pdl(argmax_part_kernel, dim3(grid), dim3(256), 0, st, logits, V, key);
    if (e != cudaSuccess) return e;
    return launch_pdl(argmax_finish_kernel, dim3(1), dim3(1), 0, st, key, token, pos, out_tokens, max_tokens);
}

} // namespace b200q
