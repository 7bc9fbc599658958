// Causal prefill attention on the 5th-generation tensor cores (tcgen05,
// bf16 operands, f32 accumulation in tensor memory) -- the attention of
// engine/model.py:130-160 (forward_sequence) for the batched prompt: query row
// t (position *pos + t, RoPE already applied) attends to cache positions
// 0 .. *pos + t of its KV head (grouped-query: head h reads KV head
// h / (H / KV)), softmax(q k^T / sqrt(hd)) v.
//
// Two launches:
//   attn_stage_bf16_kernel  bf16 copies of the rotated queries [T][H*hd] and of
//                           the layer's K/V cache rows [0, *pos + T) (rows up
//                           to the next multiple of 128 zero-filled), so that
//                           TMA can feed the tensor cores;
//   attn_prefill_tc_kernel  one CTA per (head, 128-query block), heaviest
//                           (latest) blocks first, flash-attention style over
//                           128-key blocks:
//     warp 0      TMA: Q once (two 64-dim SW128 boxes), K and V blocks
//                 double-buffered;
//     warp 1      TMEM allocation; lane 0 issues S(j) = Q K(j)^T (M = N = 128,
//                 K = hd) into one of two S accumulators, then O += P(j) V(j)
//                 (A = P from shared memory, K-major; B = V, MN-major: the TMA
//                 rows of V are keys, its 64-dim boxes the N atoms), S(j+1)
//                 issued before O += P(j) V(j) so that the tensor pipe works
//                 while the softmax warps handle S(j);
//     warps 4-7   one query row per thread (the row's TMEM lane): S row from
//                 TMEM, causal mask, running max in the log2 domain, O
//                 rescaled in TMEM when the max grows, P = exp2(s - m) as bf16
//                 into the SW128 K-major P tile; at the end O / l -> bf16.
// Every wait is bounded (error word, then the CTA leaves).  hd = 128.
#include "common.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <cmath>

namespace b200q {

cudaError_t make_map_bf16(CUtensorMap *m, const void *ptr, long long rows, long long cols, int box_rows);

constexpr int FA_B = 128;                   // queries per CTA = keys per block
constexpr int FA_HD = 128;                  // head dim
constexpr int FA_THREADS = 256;
constexpr int FA_TILE = FA_B * 64 * 2;      // 16 KB: 128 rows x 64 bf16 (one 128-byte swizzle column)

// ---------------------------------------------------------------- staging
__global__ void __launch_bounds__(256) attn_stage_bf16_kernel(const float *__restrict__ qkv,
                                                              const float *__restrict__ kc,
                                                              const float *__restrict__ vc,
                                                              const int *__restrict__ pos_p, int T, int H, int KV,
                                                              int hd, int max_seq, __nv_bfloat16 *__restrict__ qb,
                                                              __nv_bfloat16 *__restrict__ kb,
                                                              __nv_bfloat16 *__restrict__ vb, int *err)
{
    pdl_enter();
    const int p0 = *pos_p;
    if (p0 < 0 || p0 + T > max_seq) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ERR_BAD_INDEX);
        return;
    }
    const long long qd4 = (long long)H * hd / 4, kd4 = (long long)KV * hd / 4;
    const long long R4 = (long long)(H + 2 * KV) * hd / 4;
    const int filled = p0 + T;
    const int rows = min(max_seq, (filled + FA_B - 1) / FA_B * FA_B);
    const long long nq = (long long)T * qd4, nkv = (long long)rows * kd4;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nq + nkv; i += stride) {
        if (i < nq) {
            const long long t = i / qd4, c = i - t * qd4;
            const float4 v = __ldg(reinterpret_cast<const float4 *>(qkv) + t * R4 + c);
            const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
            *reinterpret_cast<uint2 *>(qb + 4 * i) = make_uint2(*reinterpret_cast<const uint32_t *>(&lo),
                                                                *reinterpret_cast<const uint32_t *>(&hi));
        } else {
            const long long j = i - nq, r = j / kd4;
            const bool live = r < filled;
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 kv = live ? __ldg(reinterpret_cast<const float4 *>(kc) + j) : zero;
            const float4 vv = live ? __ldg(reinterpret_cast<const float4 *>(vc) + j) : zero;
            const __nv_bfloat162 k0 = __floats2bfloat162_rn(kv.x, kv.y), k1 = __floats2bfloat162_rn(kv.z, kv.w);
            const __nv_bfloat162 v0 = __floats2bfloat162_rn(vv.x, vv.y), v1 = __floats2bfloat162_rn(vv.z, vv.w);
            *reinterpret_cast<uint2 *>(kb + 4 * j) = make_uint2(*reinterpret_cast<const uint32_t *>(&k0),
                                                                *reinterpret_cast<const uint32_t *>(&k1));
            *reinterpret_cast<uint2 *>(vb + 4 * j) = make_uint2(*reinterpret_cast<const uint32_t *>(&v0),
                                                                *reinterpret_cast<const uint32_t *>(&v1));
        }
    }
}

// ---------------------------------------------------------------- helpers
// Shared-memory descriptor of an MN-major operand in 128-byte swizzle atoms:
// 8 K-rows of 128 bytes (64 MN elements) per atom, the next 8 K-rows
// ``sbo`` bytes on, the next 64 MN elements ``lbo`` bytes on.
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t smem, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = 0;
    d |= (uint64_t)((smem & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x on the special-function unit (PTX ex2.approx; a few ulp, far below the
// bf16 rounding of the probabilities it feeds).
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------- kernel
// Shared layout (1024-aligned): Q [2 tiles] | K [2 stages x 2 tiles] |
// V [2 stages x 2 tiles] | P [2 tiles] | barriers | TMEM address.
// Tensor memory: S accumulators at columns 0 and 128, O at 256.
__global__ void __launch_bounds__(FA_THREADS, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                           const __grid_constant__ CUtensorMap map_v, const int *__restrict__ pos_p, int T, int H,
                           int KV, int max_seq, float scale_log2, __nv_bfloat16 *__restrict__ out, int *err)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
    const uint32_t sQ = base, sK = sQ + 2 * FA_TILE, sV = sK + 4 * FA_TILE, sP = sV + 4 * FA_TILE;
    const uint32_t sBar = sP + 2 * FA_TILE;
    const uint32_t q_full = sBar, k_full = q_full + 8, v_full = k_full + 16, k_empty = v_full + 16,
                   v_empty = k_empty + 16, s_full = v_empty + 16, s_empty = s_full + 16, p_full = s_empty + 16,
                   pv_done = p_full + 8, o_full = pv_done + 8, tmem_slot = o_full + 8;

    pdl_enter();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, qblk = gridDim.y - 1 - blockIdx.y, t0 = qblk * FA_B;
    const int g = h / (H / KV);
    const int p0 = *pos_p;
    if (p0 < 0 || p0 + T > max_seq || t0 >= T) return;       // reported by the staging kernel; CTA-uniform
    const int q_rows = min(FA_B, T - t0);
    const int nkv = (p0 + t0 + q_rows - 1) / FA_B + 1;        // key blocks this query block sees

    if (tid == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(k_full + 8 * s, 1);
            mbar_init(v_full + 8 * s, 1);
            mbar_init(k_empty + 8 * s, 1);
            mbar_init(v_empty + 8 * s, 1);
            mbar_init(s_full + 8 * s, 1);
            mbar_init(s_empty + 8 * s, 4);
        }
        mbar_init(p_full, 4);
        mbar_init(pv_done, 1);
        mbar_init(o_full, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = lds32(tmem_slot);
    bool ok = true;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, 2 * FA_TILE);
            tma_load_2d(sQ, &map_q, h * FA_HD, t0, q_full);
            tma_load_2d(sQ + FA_TILE, &map_q, h * FA_HD + 64, t0, q_full);
            for (int j = 0; j < nkv && ok; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(k_empty + 8 * s, ((j >> 1) - 1) & 1, err)) { ok = false; break; }
                mbar_arrive_expect_tx(k_full + 8 * s, 2 * FA_TILE);
                tma_load_2d(sK + s * 2 * FA_TILE, &map_k, g * FA_HD, j * FA_B, k_full + 8 * s);
                tma_load_2d(sK + s * 2 * FA_TILE + FA_TILE, &map_k, g * FA_HD + 64, j * FA_B, k_full + 8 * s);
                if (j >= 2 && !mbar_wait(v_empty + 8 * s, ((j >> 1) - 1) & 1, err)) { ok = false; break; }
                mbar_arrive_expect_tx(v_full + 8 * s, 2 * FA_TILE);
                tma_load_2d(sV + s * 2 * FA_TILE, &map_v, g * FA_HD, j * FA_B, v_full + 8 * s);
                tma_load_2d(sV + s * 2 * FA_TILE + FA_TILE, &map_v, g * FA_HD + 64, j * FA_B, v_full + 8 * s);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t id_s = idesc_bf16(FA_B, FA_B);                  // A, B K-major
            const uint32_t id_pv = idesc_bf16(FA_B, FA_HD) | (1u << 16);   // B (V) MN-major
            auto issue_s = [&](int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(k_full + 8 * s, (j >> 1) & 1, err)) return false;
                if (j >= 2 && !mbar_wait(s_empty + 8 * s, ((j >> 1) - 1) & 1, err)) return false;
                tc_fence_after();
                const uint32_t kbase = sK + s * 2 * FA_TILE;
#pragma unroll
                for (int kk = 0; kk < FA_HD / 16; ++kk) {
                    const uint32_t off = (uint32_t)((kk >> 2) * FA_TILE + (kk & 3) * 32);
                    umma_bf16(tmem + (uint32_t)(s * FA_B), sw128_desc(sQ + off), sw128_desc(kbase + off), id_s,
                              kk > 0 ? 1u : 0u);
                }
                umma_commit(s_full + 8 * s);
                umma_commit(k_empty + 8 * s);
                return true;
            };
            ok = mbar_wait(q_full, 0, err) && issue_s(0);
            for (int j = 0; j < nkv && ok; ++j) {
                if (j + 1 < nkv && !issue_s(j + 1)) { ok = false; break; }
                const int s = j & 1;
                if (!mbar_wait(p_full, j & 1, err) || !mbar_wait(v_full + 8 * s, (j >> 1) & 1, err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t vbase = sV + s * 2 * FA_TILE;
#pragma unroll
                for (int kk = 0; kk < FA_B / 16; ++kk) {
                    const uint32_t aoff = (uint32_t)((kk >> 2) * FA_TILE + (kk & 3) * 32);
                    umma_bf16(tmem + 2u * FA_B, sw128_desc(sP + aoff),
                              sw128_mn_desc(vbase + (uint32_t)kk * 2048u, FA_TILE, 1024), id_pv,
                              (j > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(pv_done);
                umma_commit(v_empty + 8 * s);
            }
            if (ok) umma_commit(o_full);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax / epilogue: row q of the block
        const int quarter = warp - 4, q = quarter * 32 + lane;
        const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
        const int qpos = p0 + t0 + q;
        float m = -INFINITY, l = 0.f;
        for (int j = 0; j < nkv; ++j) {
            const int s = j & 1;
            if (!mbar_wait(s_full + 8 * s, (j >> 1) & 1, err)) { ok = false; break; }
            tc_fence_after();
            uint32_t sv[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_addr + (uint32_t)(s * FA_B + 32 * c), sv[c]);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_empty + 8 * s);                    // S buffer may be overwritten
            // scaled scores (log2 domain), causal mask, block max
            const int key0 = j * FA_B;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float x = key0 + 32 * c + i <= qpos ? __uint_as_float(sv[c][i]) * scale_log2 : -INFINITY;
                    sv[c][i] = __float_as_uint(x);
                    mx = fmaxf(mx, x);
                }
            const float m_new = fmaxf(m, mx);
            // O and the P tile are free once the previous P V product has completed
            if (j > 0 && !mbar_wait(pv_done, (j - 1) & 1, err)) { ok = false; break; }
            tc_fence_after();
            if (j > 0 && __any_sync(0xffffffffu, m_new > m)) {
                const float alpha = m_new > m ? fast_exp2(m - m_new) : 1.0f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_addr + (uint32_t)(2 * FA_B + 32 * c), o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tmem + lane_addr + (uint32_t)(2 * FA_B + 32 * c), o);
                }
                tmem_st_wait();
                l *= alpha;
            }
            m = m_new;
            // P = exp2(x - m) as bf16 into row q of the K-major SW128 P tile (16 chunks of 8 keys)
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
                for (int k8 = 0; k8 < 4; ++k8) {
                    uint32_t pk[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float a = fast_exp2(__uint_as_float(sv[c][8 * k8 + 2 * e]) - m);
                        const float b = fast_exp2(__uint_as_float(sv[c][8 * k8 + 2 * e + 1]) - m);
                        l += a + b;
                        pk[e] = pack_bf16(a, b);
                    }
                    const int kc = 4 * c + k8;                          // key chunk 0..15
                    const uint32_t dst = sP + (uint32_t)((kc >> 3) * FA_TILE + q * 128) +
                                         ((((uint32_t)kc & 7u) ^ ((uint32_t)q & 7u)) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(pk[0]), "r"(pk[1]),
                                 "r"(pk[2]), "r"(pk[3])
                                 : "memory");
                }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        // epilogue: O / l -> bf16 row t0 + q
        if (ok && mbar_wait(o_full, 0, err)) {
            tc_fence_after();
            const float inv = 1.0f / l;
            const bool live = q < q_rows;
            __nv_bfloat16 *dst = out + (long long)(t0 + q) * H * FA_HD + (long long)h * FA_HD;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t o[32];
                tmem_ld32(tmem + lane_addr + (uint32_t)(2 * FA_B + 32 * c), o);
                tmem_ld_wait();
                if (live) {
#pragma unroll
                    for (int k8 = 0; k8 < 4; ++k8) {
                        uint4 w;
                        w.x = pack_bf16(__uint_as_float(o[8 * k8]) * inv, __uint_as_float(o[8 * k8 + 1]) * inv);
                        w.y = pack_bf16(__uint_as_float(o[8 * k8 + 2]) * inv, __uint_as_float(o[8 * k8 + 3]) * inv);
                        w.z = pack_bf16(__uint_as_float(o[8 * k8 + 4]) * inv, __uint_as_float(o[8 * k8 + 5]) * inv);
                        w.w = pack_bf16(__uint_as_float(o[8 * k8 + 6]) * inv, __uint_as_float(o[8 * k8 + 7]) * inv);
                        *reinterpret_cast<uint4 *>(dst + 32 * c + 8 * k8) = w;
                    }
                }
            }
        }
        tc_fence_before();
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------- host side
constexpr size_t FA_SMEM = 1024 + 14 * (size_t)FA_TILE + 256;

size_t attn_prefill_tc_scratch_bytes(int T, int H, int KV, int hd, int max_seq)
{
    return ((size_t)T * H * hd + 2 * (size_t)max_seq * KV * hd) * sizeof(__nv_bfloat16) + 256;
}

cudaError_t launch_attn_prefill_tc(const float *qkv, const float *kc, const float *vc, const int *pos, int T, int H,
                                   int KV, int hd, int max_seq, void *scratch, size_t scratch_bytes,
                                   __nv_bfloat16 *out, int *err, int num_sms, cudaStream_t st)
{
    if (T < 1 || H < 1 || KV < 1 || H % KV || hd != FA_HD || max_seq < 1 || !scratch ||
        scratch_bytes < attn_prefill_tc_scratch_bytes(T, H, KV, hd, max_seq) ||
        (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(kc) & 15) ||
        (reinterpret_cast<uintptr_t>(vc) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
        (reinterpret_cast<uintptr_t>(scratch) & 15))
        return cudaErrorInvalidValue;
    __nv_bfloat16 *qb = static_cast<__nv_bfloat16 *>(scratch);
    __nv_bfloat16 *kb = qb + (size_t)T * H * hd;
    __nv_bfloat16 *vb = kb + (size_t)max_seq * KV * hd;
    CUtensorMap mq, mk, mv;
    cudaError_t e = make_map_bf16(&mq, qb, T, (long long)H * hd, FA_B);
    if (e == cudaSuccess) e = make_map_bf16(&mk, kb, max_seq, (long long)KV * hd, FA_B);
    if (e == cudaSuccess) e = make_map_bf16(&mv, vb, max_seq, (long long)KV * hd, FA_B);
    if (e != cudaSuccess) return e;
    const long long work4 = ((long long)T * H * hd + (long long)max_seq * KV * hd) / 4;
    const int grid_stage = (int)std::min<long long>((work4 + 255) / 256, (long long)num_sms * 8);
    e = launch_pdl(attn_stage_bf16_kernel, dim3(grid_stage), dim3(256), 0, st, qkv, kc, vc, pos, T, H, KV, hd,
                   max_seq, qb, kb, vb, err);
    if (e != cudaSuccess) return e;
    static bool attr = false;
    if (!attr) {
        e = cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FA_SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)hd);
    return launch_pdl(attn_prefill_tc_kernel, dim3(H, (T + FA_B - 1) / FA_B), dim3(FA_THREADS), FA_SMEM, st, mq, mk,
                      mv, pos, T, H, KV, max_seq, scale_log2, out, err);
}

} // namespace b200q
