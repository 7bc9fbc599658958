// ZAYA router chain and skip route (engine/zaya.py:274-307, ZayaModel._moe),
// batched over tokens.  The router projections themselves are f32 linear
// layers (moe_router_kernel); this file holds the element/row-wise steps:
//   router += prev_router * w_eda                      (EDA, zaya.py:283-284)
//   state = router; router = rmsnorm(router) * norm_w  (zaya.py:285-286,
//                                                       model.py:82)
//   gelu(x) = x * (1 + erf(x / sqrt 2)) / 2            (zaya.py:181-186, exact)
// and the copy that serves the learned skip route (expert index E): the
// slot's output row is the block input row itself (zaya.py:297-301).
#include "common.cuh"

namespace b200q {

// One CTA per token row; fixed-order block reduction (deterministic).
__global__ void __launch_bounds__(256) zaya_router_prep_kernel(const float *__restrict__ x, const float *__restrict__ prev,
                                                               const float *__restrict__ w_eda,
                                                               const float *__restrict__ norm_w, int R, float eps,
                                                               float *__restrict__ state, float *__restrict__ out)
{
    __shared__ float red[256];
    const long long t = blockIdx.x;
    const float *xr = x + t * R;
    float ss = 0.f;
    for (int i = threadIdx.x; i < R; i += blockDim.x) {
        float v = xr[i];
        if (prev && w_eda) v = v + prev[t * R + i] * w_eda[i];
        state[t * R + i] = v;
        ss = fmaf(v, v, ss);
    }
    red[threadIdx.x] = ss;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
        if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
        __syncthreads();
    }
    const float inv = 1.0f / sqrtf(red[0] / (float)R + eps);
    for (int i = threadIdx.x; i < R; i += blockDim.x) out[t * R + i] = state[t * R + i] * inv * norm_w[i];
}

__global__ void gelu_kernel(float *__restrict__ x, long long n)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        x[i] = v * (1.0f + erff(v / 1.41421356237309515f)) * 0.5f;
    }
}

// dst rows [offsets[g], offsets[g+1]) = src rows (bf16, D columns); at most
// max_rows rows are visited.
__global__ void copy_rows_range_kernel(const __nv_bfloat16 *__restrict__ src, __nv_bfloat16 *__restrict__ dst,
                                       const int *__restrict__ offsets, int g, int D, int max_rows)
{
    const int a = offsets[g], b = offsets[g + 1];
    for (int r = a + blockIdx.x; r < b && r < max_rows; r += gridDim.x) {
        const uint4 *s = reinterpret_cast<const uint4 *>(src + (long long)r * D);
        uint4 *d = reinterpret_cast<uint4 *>(dst + (long long)r * D);
        for (int c = threadIdx.x; c < D / 8; c += blockDim.x) d[c] = s[c];
    }
}

cudaError_t launch_zaya_router_prep(const float *x, const float *prev, const float *w_eda, const float *norm_w, int T,
                                    int R, float eps, float *state, float *out, cudaStream_t st)
{
    if (T < 1 || R < 1) return cudaErrorInvalidValue;
    zaya_router_prep_kernel<<<T, 256, 0, st>>>(x, prev, w_eda, norm_w, R, eps, state, out);
    return cudaGetLastError();
}

cudaError_t launch_gelu(float *x, long long n, int num_sms, cudaStream_t st)
{
    if (n < 1) return cudaErrorInvalidValue;
    long long blocks = (n + 255) / 256;
    if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
    gelu_kernel<<<(int)blocks, 256, 0, st>>>(x, n);
    return cudaGetLastError();
}

cudaError_t launch_copy_rows_range(const void *src, void *dst, const int *offsets, int g, int D, int max_rows,
                                   int num_sms, cudaStream_t st)
{
    if (D < 8 || D % 8 || max_rows < 1 || (reinterpret_cast<uintptr_t>(src) & 15) ||
        (reinterpret_cast<uintptr_t>(dst) & 15))
        return cudaErrorInvalidValue;
    copy_rows_range_kernel<<<2 * num_sms, 128, 0, st>>>(static_cast<const __nv_bfloat16 *>(src),
                                                         static_cast<__nv_bfloat16 *>(dst), offsets, g, D, max_rows);
    return cudaGetLastError();
}

} // namespace b200q
