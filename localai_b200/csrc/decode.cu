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

namespace b200q {

constexpr int ATT_CHUNK = 128;

// x += delta (when given); h = x / sqrt(mean(x^2) + eps) * w  (engine/model.py:82)
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(float *__restrict__ x, const float *__restrict__ delta,
                                                          const float *__restrict__ w, int D, float eps,
                                                          float *__restrict__ h)
{
    __shared__ float red[256];
    const long long t = blockIdx.x;
    float *xr = x + t * D;
    float ss = 0.f;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v = xr[i];
        if (delta) {
            v = v + delta[t * D + i];
            xr[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    red[threadIdx.x] = ss;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    const float inv = 1.0f / sqrtf(red[0] / (float)D + eps);
    for (int i = threadIdx.x; i < D; i += blockDim.x) h[t * D + i] = xr[i] * inv * w[i];
}

// qkv = [q (H*hd) | k (KV*hd) | v (KV*hd)]: rotate q and k in place over the
// first ``rotary`` dims (adjacent pairs, engine/model.py:205-217):
// inv_j = 1 / base^(j / half), angle = pos * inv_j.
__global__ void rope_kernel(float *__restrict__ qkv, int H, int KV, int hd, int rotary, float base,
                            const int *__restrict__ pos_p, int max_seq, int *err)
{
    const int pos = *pos_p;
    if (pos < 0 || pos >= max_seq) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ERR_BAD_INDEX);
        return;
    }
    const int half = rotary / 2;
    const int pairs = (H + KV) * half;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < pairs; i += gridDim.x * blockDim.x) {
        const int hh = i / half, j = i % half;
        const float inv = 1.0f / powf(base, (float)j / (float)half);
        const float ang = (float)pos * inv;
        const float c = cosf(ang), s = sinf(ang);
        float *a = qkv + (long long)hh * hd + 2 * j;
        const float e = a[0], o = a[1];
        a[0] = e * c - o * s;
        a[1] = e * s + o * c;
    }
}

// cache[pos] = k, v (cache layout [max_seq][KV][hd], as the reference's KVCache)
__global__ void kv_store_kernel(const float *__restrict__ qkv, int H, int KV, int hd, const int *__restrict__ pos_p,
                                float *__restrict__ kc, float *__restrict__ vc, int max_seq)
{
    const int pos = *pos_p;
    if (pos < 0 || pos >= max_seq) return;
    const int n = KV * hd;
    const float *k = qkv + (long long)H * hd, *v = k + n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        kc[(long long)pos * n + i] = k[i];
        vc[(long long)pos * n + i] = v[i];
    }
}

// One CTA per (KV head g, chunk c of positions).  Scores of the G = H/KV query
// heads of group g over positions [c*ATT_CHUNK, min(pos+1, ...)); writes the
// chunk's max, sum of exp and exp-weighted V per query head.
__global__ void __launch_bounds__(128) attn_chunk_kernel(const float *__restrict__ q, const float *__restrict__ kc,
                                                         const float *__restrict__ vc, const int *__restrict__ pos_p,
                                                         int H, int KV, int hd, int max_seq,
                                                         float *__restrict__ part)
{
    extern __shared__ float asm_[];
    const int G = H / KV, g = blockIdx.x, c = blockIdx.y;
    const int L = min(*pos_p + 1, max_seq);
    const int l0 = c * ATT_CHUNK, l1 = min(L, l0 + ATT_CHUNK);
    const int nch = gridDim.y;
    // part layout: [H][nch][hd + 2]: acc[hd], max, sum
    float *qs = asm_;                         // [G][hd]
    float *sc = qs + G * hd;                  // [G][ATT_CHUNK]
    __shared__ float red[128];
    const int tid = threadIdx.x;
    for (int i = tid; i < G * hd; i += blockDim.x) qs[i] = q[(long long)g * G * hd + i];
    __syncthreads();
    const float rs = sqrtf((float)hd);
    // scores: one position per thread
    for (int l = l0 + tid; l < l0 + ATT_CHUNK; l += blockDim.x) {
        if (l < l1) {
            const float *kr = kc + ((long long)l * KV + g) * hd;
            for (int j = 0; j < G; ++j) {
                float d = 0.f;
                for (int e = 0; e < hd; ++e) d = fmaf(qs[j * hd + e], kr[e], d);
                sc[j * ATT_CHUNK + (l - l0)] = d / rs;
            }
        } else {
            for (int j = 0; j < G; ++j) sc[j * ATT_CHUNK + (l - l0)] = -INFINITY;
        }
    }
    __syncthreads();
    for (int j = 0; j < G; ++j) {
        // chunk max and sum of exp (fixed-order tree)
        float m = -INFINITY;
        for (int l = tid; l < ATT_CHUNK; l += blockDim.x) m = fmaxf(m, sc[j * ATT_CHUNK + l]);
        red[tid] = m;
        __syncthreads();
        for (int o = blockDim.x / 2; o > 0; o >>= 1) {
            if (tid < o) red[tid] = fmaxf(red[tid], red[tid + o]);
            __syncthreads();
        }
        m = red[0];
        __syncthreads();
        float s = 0.f;
        for (int l = tid; l < ATT_CHUNK; l += blockDim.x) {
            const float e = (l0 + l < l1) ? expf(sc[j * ATT_CHUNK + l] - m) : 0.f;
            sc[j * ATT_CHUNK + l] = e;
            s += e;
        }
        red[tid] = s;
        __syncthreads();
        for (int o = blockDim.x / 2; o > 0; o >>= 1) {
            if (tid < o) red[tid] += red[tid + o];
            __syncthreads();
        }
        float *pp = part + ((long long)(g * G + j) * nch + c) * (hd + 2);
        if (tid == 0) {
            pp[hd] = l1 > l0 ? m : -INFINITY;
            pp[hd + 1] = l1 > l0 ? red[0] : 0.f;
        }
        __syncthreads();
        for (int d = tid; d < hd; d += blockDim.x) {
            float a = 0.f;
            for (int l = l0; l < l1; ++l) a = fmaf(sc[j * ATT_CHUNK + (l - l0)], vc[((long long)l * KV + g) * hd + d], a);
            pp[d] = a;
        }
        __syncthreads();
    }
}

// out[h][d] = sum_c exp(m_c - M) acc_c[d] / sum_c exp(m_c - M) s_c, chunks in order.
__global__ void attn_combine_kernel(const float *__restrict__ part, int nch, int hd, float *__restrict__ out)
{
    const int h = blockIdx.x;
    const float *ph = part + (long long)h * nch * (hd + 2);
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, ph[c * (hd + 2) + hd]);
    float S = 0.f;
    for (int c = 0; c < nch; ++c) {
        const float mc = ph[c * (hd + 2) + hd];
        if (mc != -INFINITY) S += expf(mc - M) * ph[c * (hd + 2) + hd + 1];
    }
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float a = 0.f;
        for (int c = 0; c < nch; ++c) {
            const float mc = ph[c * (hd + 2) + hd];
            if (mc != -INFINITY) a += expf(mc - M) * ph[c * (hd + 2) + d];
        }
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
                               cudaStream_t st)
{
    if (T < 1 || D < 1) return cudaErrorInvalidValue;
    add_rmsnorm_kernel<<<T, 256, 0, st>>>(x, delta, w, D, eps, h);
    return cudaGetLastError();
}

cudaError_t launch_rope_kv(float *qkv, int H, int KV, int hd, int rotary, float base, const int *pos, float *kc,
                           float *vc, int max_seq, int *err, cudaStream_t st)
{
    if (H < 1 || KV < 1 || H % KV || hd < 2 || rotary < 0 || rotary > hd || rotary % 2 || max_seq < 1)
        return cudaErrorInvalidValue;
    const int pairs = (H + KV) * (rotary / 2);
    if (pairs > 0) rope_kernel<<<(pairs + 255) / 256, 256, 0, st>>>(qkv, H, KV, hd, rotary, base, pos, max_seq, err);
    kv_store_kernel<<<(KV * hd + 255) / 256, 256, 0, st>>>(qkv, H, KV, hd, pos, kc, vc, max_seq);
    return cudaGetLastError();
}

size_t attn_scratch_floats(int H, int hd, int max_seq)
{
    const int nch = (max_seq + ATT_CHUNK - 1) / ATT_CHUNK;
    return (size_t)H * nch * (hd + 2);
}

cudaError_t launch_attn_decode(const float *q, const float *kc, const float *vc, const int *pos, int H, int KV, int hd,
                               int max_seq, float *part, float *out, cudaStream_t st)
{
    if (H < 1 || KV < 1 || H % KV || hd < 1 || max_seq < 1) return cudaErrorInvalidValue;
    const int G = H / KV, nch = (max_seq + ATT_CHUNK - 1) / ATT_CHUNK;
    const size_t smem = (size_t)(G * hd + G * ATT_CHUNK) * sizeof(float);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    attn_chunk_kernel<<<dim3(KV, nch), 128, smem, st>>>(q, kc, vc, pos, H, KV, hd, max_seq, part);
    attn_combine_kernel<<<H, 128, 0, st>>>(part, nch, hd, out);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float *logits, int V, int *token, int *pos, int *out_tokens, int max_tokens,
                          cudaStream_t st)
{
    if (V < 1) return cudaErrorInvalidValue;
    argmax_kernel<<<1, 1024, 0, st>>>(logits, V, token, pos, out_tokens, max_tokens);
    return cudaGetLastError();
}

} // namespace b200q
