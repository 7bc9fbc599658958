// Batch-1 Q4_K GEMV on the integer tensor cores (sm_100a).
//
// y[r] = sum_c W[r, c] * x[c] for W = raw GGUF Q4_K rows -- localai_q4k_matvec
// (engine/native_quant.cpp:183-231, exported at :719-725), at f32-level
// accuracy: x is quantised per 256-value super-block to 16-bit fixed point
// (two signed byte planes, xq = 256*hi + lo, |xq| <= 32639, grid step
// max|x| / 32639), and every 4-bit x 8-bit product sum is exact in int32.
//
// Why tensor cores for a memory-bound GEMV: on the CUDA cores the unpacking
// and dp4a products cost more instruction issue per weight byte than HBM
// delivers per SM.  Here one mma.sync m16n8k32 (u8 x s8 -> s32) consumes 16
// rows x 32 values of one sub-block, so the CUDA cores only mask nibbles and
// apply each (row, sub-block)'s scale -- once, in exactly one thread.
//
// Fragment plan (per warp, 16 weight rows x one super-block):
//   A  = the 16 rows' qs bytes of sub-block pair p (ldmatrix.x4, identity k
//        mapping); low nibbles (& 0x0F) feed sub-block 2p, high nibbles
//        (& 0xF0, i.e. 16*q) feed sub-block 2p+1;
//   B  = 8 columns: sub-blocks 0-3 (set E) or 4-7 (set F) x {hi, lo} plane:
//        column 2i + plane of mma s is nonzero only when i == s % 4, so the
//        four mmas of a set chain into one accumulator whose columns keep the
//        sub-blocks apart;
//   D  = thread (g, t) (g = lane / 4, t = lane % 4) receives the hi and lo
//        sums of sub-blocks t (set E) and t + 4 (set F) for rows g and g + 8:
//        it alone applies those four (row, sub-block) scales.
// Sub-block scale/min decoding follows engine/dequant.py:97-120:
//   g < 4: sc = s[g] & 63, mn = s[g+4] & 63;
//   g >= 4: sc = (s[g+4] & 15) | (s[g-4] >> 6) << 4, mn = (s[g+4] >> 4) | (s[g] >> 6) << 4;
//   value = d * sc * q - dmin * mn.
//
// Pipeline: no producer warp.  A CTA takes a contiguous range of 16-row
// tiles; its 8 warps split every tile's columns (warp w owns super-blocks
// w*spw .. w*spw + spw - 1 of each chunk of 8*spw), so together they stream
// whole contiguous rows.  Each warp fetches its own [16 rows x spw super-
// blocks] pieces with one 2-D TMA copy per piece into a private ring of
// shared-memory stages (completion on a per-stage mbarrier), the ring filled
// before the programmatic-dependency wait so the weights stream while the
// previous kernel finishes.  The TMA box is spw*144 bytes wide, widened by 16
// when that is an even multiple of 16, so rows sit an odd multiple of 16
// bytes apart and ldmatrix / header loads are bank-conflict free (the extra
// 16 bytes are never used; past the row end they read as zero).  The 8 warps'
// partial row sums of a tile are added in a fixed order by whichever warp
// finishes the tile last (a shared-memory counter; no CTA-wide barrier).
// Two CTAs fit per SM (by default both from one launch: more warps hide more
// latency; with one per SM the other slot runs the next launch's stream).
#include "common.cuh"

#include <cuda.h>

namespace b200q {

cudaError_t make_map_u16_rows(CUtensorMap *m, const void *ptr, long long rows, long long row_bytes, int box_bytes,
                              int box_rows);

constexpr int GM_NW = 8;                  // warps per CTA (each owns a column slot)
constexpr int GM_THREADS = GM_NW * 32;
constexpr int GM_SB = 144;                // bytes per Q4_K super-block
constexpr float GM_XQ = 32639.0f;         // largest |xq|: 256 * 127 + 127

struct GemvMmaArgs {
    float *y;
    const float *x;
    long long ys_r;
    int rows, nsb;             // rows; super-blocks per row (cols / 256)
    int spw;                   // super-blocks per warp per chunk
    int nchunk;                // chunks per row (each GM_NW * spw super-blocks)
    int pitch;                 // shared bytes between the rows of a stage (= TMA box width)
    int stages;                // ring depth per warp
    int max_tiles;             // tiles per CTA the reduction area holds
    int *err;
};

__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&q)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3])
                 : "r"(addr));
}

__device__ __forceinline__ void sts32(uint32_t a, uint32_t v)
{
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}

__device__ __forceinline__ void gm_tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar,
                                          uint64_t pol)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(pol)
        : "memory");
}

// Quantise super-block b of x (256 values) into the B-fragment table
// xb[b][lane] (uint4 {E0, E1, F0, F1}: plane (lane/4)&1 of sub-blocks
// lane/8 and lane/8 + 4 at k-slices 4t..4t+3 and 16+4t..16+4t+3) and the
// scale table xs[b][t] (float4 {sum x of sub-block t, sum x of sub-block t+4,
// s * (t odd ? 1/16 : 1), 0}).  One warp; lane L holds values 8L .. 8L+7.
__device__ __forceinline__ void gm_quantize_sb(const float4 (&v)[2], int b, uint32_t *xbw, float *xsf, int lane)
{
    const float e[8] = {v[0].x, v[0].y, v[0].z, v[0].w, v[1].x, v[1].y, v[1].z, v[1].w};
    float m = 0.f, sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(e[i]));
#pragma unroll
    for (int i = 0; i < 8; i += 2) sum += e[i] + e[i + 1];
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);         // the four lanes of a sub-block, fixed order
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float inv = m > 0.f ? GM_XQ / m : 0.f;
    const float s = m * (1.0f / GM_XQ);
    uint32_t hi[2] = {0, 0}, lo[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = __float2int_rn(e[i] * inv);         // |q| <= 32639
        const int l = (int)(int8_t)(q & 0xff);
        const int h = (q - l) >> 8;
        lo[i >> 2] |= (uint32_t)(l & 0xff) << (8 * (i & 3));
        hi[i >> 2] |= (uint32_t)(h & 0xff) << (8 * (i & 3));
    }
    const int sbk = lane >> 2, m4 = lane & 3;              // sub-block, 8-value group inside it
    const int reg_set = sbk < 4 ? 0 : 2;
#pragma unroll
    for (int grp = 0; grp < 2; ++grp) {
        const int j = 8 * m4 + 4 * grp;                    // first value of the 4-byte group
        const int tt = j < 16 ? j >> 2 : (j - 16) >> 2;
        const int reg = reg_set + (j < 16 ? 0 : 1);
#pragma unroll
        for (int plane = 0; plane < 2; ++plane) {
            const int gg = 2 * (sbk & 3) + plane;          // column of that plane
            xbw[(b * 32 + gg * 4 + tt) * 4 + reg] = plane == 0 ? hi[grp] : lo[grp];
        }
    }
    if (m4 == 0) xsf[(b * 4 + (sbk & 3)) * 4 + (sbk < 4 ? 0 : 1)] = sum;
    if (lane < 4) xsf[(b * 4 + lane) * 4 + 2] = s * ((lane & 1) ? 0.0625f : 1.0f);
}

// Rows g and g+8 of one super-block (16 rows x 256 values at shared address
// sb, rows ``pitch`` bytes apart): the integer-tensor-core dot products with
// x's fragment table, then this thread's two sub-blocks' scales.  Adds to
// acc0 (row g) and acc1 (row g + 8).
template <int SPW>
__device__ __forceinline__ void gm_superblocks(const uint32_t (&sb)[SPW], const int (&bidx)[SPW], int nb,
                                               uint32_t pitch, uint32_t xb, uint32_t xs, int lane,
                                               const uint32_t (&msk)[4], float &acc0, float &acc1)
{
    const int g = lane >> 2, t = lane & 3, hsh = 8 * t;
    const int mrow = (lane & 7) + (lane & 8), mcol = lane & 16;
    uint4 XB[SPW];
    uint32_t q[SPW][4][4];
#pragma unroll
    for (int i = 0; i < SPW; ++i) {
        if (i < nb) {
            XB[i] = lds128(xb + (uint32_t)(bidx[i] * 32 + lane) * 16);
#pragma unroll
            for (int p = 0; p < 4; ++p) ldsm_x4(sb[i] + (uint32_t)mrow * pitch + 16 + 32 * p + mcol, q[i][p]);
        }
    }
    // four independent accumulators per super-block (pairs 0..3), two products each
    int D[SPW][4][4];
#pragma unroll
    for (int i = 0; i < SPW; ++i)
#pragma unroll
        for (int p = 0; p < 4; ++p) D[i][p][0] = D[i][p][1] = D[i][p][2] = D[i][p][3] = 0;
#pragma unroll
    for (int hn = 0; hn < 2; ++hn)               // low nibbles (sub-block 2p), then high (2p + 1)
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int i = 0; i < SPW; ++i) {
                if (i < nb) {
                    uint32_t A[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) A[r] = q[i][p][r] & (hn ? 0xF0F0F0F0u : 0x0F0F0F0Fu);
                    const uint32_t m = msk[(2 * p + hn) & 3];
                    const uint32_t b0 = p < 2 ? XB[i].x : XB[i].z, b1 = p < 2 ? XB[i].y : XB[i].w;
                    mma_u8s8(D[i][p], A, b0 & m, b1 & m);
                }
            }
#pragma unroll
    for (int i = 0; i < SPW; ++i) {
        if (i < nb) {
            // set E = pairs 0, 1 (sub-blocks 0-3); set F = pairs 2, 3 (4-7): disjoint columns, exact sum
            int E[4], F[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                E[r] = D[i][0][r] + D[i][1][r];
                F[r] = D[i][2][r] + D[i][3][r];
            }
            const uint4 XS = lds128(xs + (uint32_t)(bidx[i] * 4 + t) * 16);
            const uint4 h0 = lds128(sb[i] + (uint32_t)g * pitch);
            const uint4 h8 = lds128(sb[i] + (uint32_t)(g + 8) * pitch);
            // scales of sub-blocks t and t + 4 (engine/dequant.py:108-113)
            const float sx = __uint_as_float(XS.z), xs_t = __uint_as_float(XS.x), xs_t4 = __uint_as_float(XS.y);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const uint4 h = half ? h8 : h0;
                const int I_t = 256 * (half ? E[2] : E[0]) + (half ? E[3] : E[1]);
                const int I_t4 = 256 * (half ? F[2] : F[0]) + (half ? F[3] : F[1]);
                const uint32_t sc_t = (h.y >> hsh) & 63u, mn_t = (h.z >> hsh) & 63u;
                const uint32_t sc_t4 = ((h.w >> hsh) & 15u) | (((h.y >> hsh) >> 6 & 3u) << 4);
                const uint32_t mn_t4 = ((h.w >> hsh) >> 4 & 15u) | (((h.z >> hsh) >> 6 & 3u) << 4);
                const float d = h2f(h.x) * sx, dmin = h2f(h.x >> 16);
                float v = fmaf(d * (float)sc_t, (float)I_t, d * (float)sc_t4 * (float)I_t4);
                v = fmaf(-dmin, fmaf((float)mn_t, xs_t, (float)mn_t4 * xs_t4), v);
                if (half) acc1 += v; else acc0 += v;
            }
        }
    }
}

// Shared layout: [mbarriers GM_NW x stages][tile counters][partials max_tiles x 16 x GM_NW]
// [x tables: nsb x 512 B + nsb x 64 B][rings: GM_NW x stages x 16 x pitch] (128-B aligned).
template <int SPW>
__global__ void __launch_bounds__(GM_THREADS, 2) gemv_q4k_mma_kernel(const __grid_constant__ CUtensorMap map,
                                                                     const GemvMmaArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t sbase = smem_addr(smem);
    const uint32_t bars = sbase + (uint32_t)(warp * a.stages) * 8;
    int *cnt = reinterpret_cast<int *>(smem + GM_NW * a.stages * 8);
    float *red = reinterpret_cast<float *>(cnt + a.max_tiles);
    const uint32_t xb = (smem_addr(red + a.max_tiles * 16 * GM_NW) + 15) & ~15u;     // [nsb][32] uint4
    const uint32_t xs = xb + (uint32_t)a.nsb * 512;                                   // [nsb][4] float4
    const uint32_t stage_bytes = (uint32_t)(16 * a.pitch);
    const uint32_t ring = ((xs + (uint32_t)a.nsb * 64 + 127) & ~127u) + (uint32_t)warp * a.stages * stage_bytes;

    // this CTA's 16-row tiles; a warp's stages run tile-major, chunk-minor
    const int tiles = (a.rows + 15) / 16;
    const int t_begin = (int)((long long)blockIdx.x * tiles / gridDim.x);
    const int t_end = (int)((long long)(blockIdx.x + 1) * tiles / gridDim.x);
    const int ntl = t_end - t_begin;
    const int csb = GM_NW * SPW;
    // a warp with no super-blocks in a chunk fetches nothing for it (only the last chunk can be short)
    auto has_work = [&](int c) { return c * csb + warp * SPW < a.nsb; };
    // issue cursor (lane 0): next stage to fetch, as (tile, chunk), and its ring slot
    int itl = 0, ic = 0, islot = 0;
    // TMA of the cursor's stage into its slot; a stage without work completes its
    // barrier phase at once, so that every use of a slot flips its phase
    auto issue_next = [&]() {
        if (itl >= ntl) return;
        const uint32_t bar = bars + 8u * (uint32_t)islot;
        if (has_work(ic)) {
            mbar_arrive_expect_tx(bar, stage_bytes);
            gm_tma_2d(ring + (uint32_t)islot * stage_bytes, &map, (ic * csb + warp * SPW) * (GM_SB / 2),
                      (t_begin + itl) * 16, bar, policy_evict_first());
        } else {
            mbar_arrive(bar);
        }
        if (++ic == a.nchunk) { ic = 0; ++itl; }
        if (++islot == a.stages) islot = 0;
    };

    if (lane == 0) {
        for (int s = 0; s < a.stages; ++s) mbar_init(bars + 8 * s, 1);
        mbar_fence_init();
    }
    __syncwarp();
    pdl_launch_dependents();
    // weights are read-only for the whole stream: fill the ring before the dependency wait
    if (lane == 0)
        for (int i = 0; i < a.stages; ++i) issue_next();

    // tile counters zeroed before any warp can finish a tile (shared memory,
    // not the previous kernel's output: done before the dependency wait)
    for (int i = threadIdx.x; i < a.max_tiles; i += GM_THREADS) cnt[i] = 0;
    __syncthreads();

    // ---- quantise x into the fragment tables (x may come from the previous kernel).
    // A warp reads only the super-blocks it owns (c * csb + warp * SPW + i of
    // every chunk c), so each warp quantises exactly those and starts on its
    // weights without waiting for the other warps.
    pdl_wait();
    const int nown = a.nchunk * SPW;
    auto owned = [&](int j) { return (j / SPW) * csb + warp * SPW + j % SPW; };
    for (int j0 = 0; j0 < nown; j0 += 4) {
        float4 v[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int b = owned(j0 + i);
            if (j0 + i < nown && b < a.nsb) {
                const float4 *p = reinterpret_cast<const float4 *>(a.x + (long long)b * 256 + 8 * lane);
                v[i][0] = __ldg(p);
                v[i][1] = __ldg(p + 1);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int b = owned(j0 + i);
            if (j0 + i < nown && b < a.nsb)                          // warp-uniform condition
                gm_quantize_sb(v[i], b, reinterpret_cast<uint32_t *>(smem + (xb - sbase)),
                               reinterpret_cast<float *>(smem + (xs - sbase)), lane);
        }
    }
    __syncwarp();

    const int g = lane >> 2, t = lane & 3;
    // selection masks: column pair i of a set belongs to sub-block i of that set
    uint32_t msk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) msk[i] = (i == (g >> 1)) ? 0xffffffffu : 0u;
    float acc0 = 0.f, acc1 = 0.f;                            // rows g and g + 8 of the current tile
    int slot = 0;
    uint32_t phase = 0;
    for (int tl = 0; tl < ntl; ++tl) {
        for (int c = 0; c < a.nchunk; ++c) {
            if (!mbar_wait(bars + 8u * (uint32_t)slot, phase, a.err)) {
                // give up: wait (bounded) for this warp's copies still in flight, then leave
                if (lane == 0) {
                    int sl = slot;
                    uint32_t ph = phase;
                    for (int j = 0; j < a.stages; ++j) {
                        mbar_wait(bars + 8u * (uint32_t)sl, ph, a.err);
                        if (++sl == a.stages) { sl = 0; ph ^= 1u; }
                    }
                }
                return;
            }
            if (has_work(c)) {
                const uint32_t base = ring + (uint32_t)slot * stage_bytes;
                const int b0 = c * csb + warp * SPW;
                const int nb = min(SPW, a.nsb - b0);
                uint32_t sb[SPW];
                int bidx[SPW];
#pragma unroll
                for (int i = 0; i < SPW; ++i) {
                    sb[i] = base + (uint32_t)i * GM_SB;
                    bidx[i] = b0 + i;
                }
                gm_superblocks<SPW>(sb, bidx, nb, (uint32_t)a.pitch, xb, xs, lane, msk, acc0, acc1);
            }
            __syncwarp();                                    // every lane is done reading the slot
            if (lane == 0) issue_next();                     // refill it
            if (++slot == a.stages) { slot = 0; phase ^= 1u; }
        }
        // tile done: this warp's partial row sums; the last of the 8 warps adds them in warp order
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        float *pr = red + tl * 16 * GM_NW;
        if (t == 0) {
            pr[g * GM_NW + warp] = acc0;
            pr[(g + 8) * GM_NW + warp] = acc1;
        }
        acc0 = acc1 = 0.f;
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&cnt[tl], 1) == GM_NW - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < 16) {
                const int row = (t_begin + tl) * 16 + lane;
                const volatile float *pp = pr + lane * GM_NW;
                float v = 0.f;
#pragma unroll
                for (int q = 0; q < GM_NW; ++q) v += pp[q];
                if (row < a.rows) a.y[row * a.ys_r] = v;
            }
        }
    }
}

// ---------------------------------------------------------------- host side
static int g_gm_spw = 0;                  // 0: choose
static int g_gm_stages = 0;               // 0: as many as fit
static int g_gm_ctas_per_sm = 2;          // CTAs of one launch per SM (1: the other slot overlaps the next launch)
void gemv_mma_set_tuning(int spw, int stages, int ctas_per_sm)
{
    if (spw >= 0 && spw <= 3) g_gm_spw = spw;
    if (stages >= 0 && stages <= 16) g_gm_stages = stages;
    if (ctas_per_sm == 1 || ctas_per_sm == 2) g_gm_ctas_per_sm = ctas_per_sm;
}

// Row pitch of a stage: spw super-blocks, widened to an odd multiple of 16 bytes.
static int gm_pitch(int spw) { return (spw * 9) % 2 ? spw * GM_SB : spw * GM_SB + 16; }

static size_t gm_fixed_smem(int nsb, int max_tiles)
{
    size_t off = (size_t)GM_NW * 16 * 8 + (size_t)max_tiles * 4 + (size_t)max_tiles * 16 * GM_NW * 4;
    off = (off + 15) / 16 * 16 + (size_t)nsb * 576;
    return (off + 127) / 128 * 128 + 128;     // + slack for the base alignment
}

constexpr size_t GM_SMEM_BUDGET = 110 * 1024;    // two CTAs per SM

template <int SPW>
static cudaError_t gm_launch(const CUtensorMap &map, const GemvMmaArgs &a, int grid, size_t smem, cudaStream_t st)
{
    static size_t attr = 0;
    if (smem > attr) {
        cudaError_t e = cudaFuncSetAttribute(gemv_q4k_mma_kernel<SPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        attr = smem;
    }
    return launch_pdl(gemv_q4k_mma_kernel<SPW>, dim3(grid), dim3(GM_THREADS), smem, st, map, a);
}

// True when this kernel takes the call (else the caller uses the general GEMV).
bool gemv_mma_supported(int type, const void *w, int rows, int cols, int tokens)
{
    if (type != T_Q4_K || tokens != 1 || rows < 1 || cols < 256 || cols % 256) return false;
    if (reinterpret_cast<uintptr_t>(w) & 15) return false;
    return gm_fixed_smem(cols / 256, 64) + 2 * GM_NW * 16 * gm_pitch(1) <= GM_SMEM_BUDGET;
}

cudaError_t launch_gemv_mma(const void *w, const float *x, float *y, long long ys_r, int rows, int cols, int *err,
                            int num_sms, cudaStream_t st)
{
    if (!gemv_mma_supported(T_Q4_K, w, rows, cols, 1) || (reinterpret_cast<uintptr_t>(x) & 15))
        return cudaErrorInvalidValue;
    GemvMmaArgs a = {};
    a.x = x;
    a.y = y;
    a.ys_r = ys_r;
    a.rows = rows;
    a.nsb = cols / 256;
    const int tiles = (rows + 15) / 16;
    int grid = num_sms * g_gm_ctas_per_sm < tiles ? num_sms * g_gm_ctas_per_sm : tiles;
    // the reduction area holds every tile of a CTA: grow the grid if that would exceed 64
    if ((tiles + grid - 1) / grid > 64) grid = (tiles + 63) / 64;
    a.max_tiles = (tiles + grid - 1) / grid;
    const size_t fixed = gm_fixed_smem(a.nsb, a.max_tiles);
    // super-blocks per warp: 2 when two such stages fit per warp, else 1
    int spw = g_gm_spw;
    if (spw == 0) spw = (a.nsb >= 2 * GM_NW && fixed + 2 * GM_NW * 16 * gm_pitch(2) <= GM_SMEM_BUDGET) ? 2 : 1;
    if (a.nsb < GM_NW * spw) spw = 1;
    a.spw = spw;
    a.nchunk = (a.nsb + GM_NW * spw - 1) / (GM_NW * spw);
    a.pitch = gm_pitch(spw);
    const size_t per_stage = (size_t)GM_NW * 16 * a.pitch;
    int stages = (int)((GM_SMEM_BUDGET - fixed) / per_stage);
    const int n_it = a.max_tiles * a.nchunk;
    if (stages > n_it) stages = n_it;                        // never more than the whole CTA slice
    if (g_gm_stages > 0 && g_gm_stages < stages) stages = g_gm_stages;
    if (stages < 1) return cudaErrorInvalidValue;
    a.stages = stages;
    a.err = err;
    const size_t smem = fixed + (size_t)stages * per_stage;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    CUtensorMap map;
    cudaError_t e = make_map_u16_rows(&map, w, rows, (long long)a.nsb * GM_SB, a.pitch, 16);
    if (e != cudaSuccess) return e;
    switch (spw) {
    case 1: return gm_launch<1>(map, a, grid, smem, st);
    case 2: return gm_launch<2>(map, a, grid, smem, st);
    default: return gm_launch<3>(map, a, grid, smem, st);
    }
}

} // namespace b200q
