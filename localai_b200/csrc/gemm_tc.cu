// Grouped GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) with the
// GGML weights dequantised inside the kernel.
//
// For every group g (an expert, or the single weight matrix of a dense
// prefill) and its M_g activation rows [row_off[g], row_off[g+1]) of a bf16
// matrix X:
//     C_g[m, n] = sum_k X[row_off[g] + m, k] * W_g[n, k]
// where W_g is stored as raw GGUF blocks (Q4_K) -- the batched path of the
// reference (engine/native_quant.cpp:620-703 decoded_matmul_row / MatmulPool,
// and the per-expert products of engine/zaya.py:303-306).
//
// Tile: 128 weight rows (MMA M) x 256 activation rows (MMA N) x the full K, in
// K-steps of 64 (one 128-byte swizzle atom of bf16).  The last tile of a group
// issues its MMAs with N = its valid rows rounded up to 16, so skewed expert
// loads do not pay for empty columns.
//
// Warp roles (512 threads, one CTA per SM, persistent over tiles):
//   warp 0        TMA: activation box [64 k x 256 rows] (SWIZZLE_128B) per
//                 K-step, raw weight boxes [one 256-value block x 64 rows] x 2
//                 per 256-K chunk;
//   warp 1        TMEM allocator; lane 0 issues tcgen05.mma (kind::f16, bf16
//                 in, f32 accumulate in TMEM; two 256-column accumulators so
//                 the epilogue of one tile overlaps the main loop of the next)
//                 and tcgen05.commit;
//   warps 4-7     epilogue: tcgen05.ld of the accumulator, then either
//                 (gate/up mode) SiLU(gate) * up -> bf16, or (plain mode) a
//                 per-row scaled f32 store;
//   warps 8-15    dequantisers: raw Q4_K block bytes (shared memory) -> bf16 A
//                 tile in the canonical K-major SWIZZLE_128B layout.
// All waits are bounded (an error word is set and the CTA leaves).
//
// Gate/up mode computes, for 64 features f0..f0+63, the 64 gate rows and the 64
// up rows of the same features in one tile, ordered so that every warp holds
// 16 gate rows and the 16 matching up rows (lanes l and l+16).
#include "common.cuh"
#include "ep.cuh"
#include "tcgen05.cuh"

#include <cuda.h>
#include <algorithm>
#include <cstring>
#include <mutex>

namespace b200q {

constexpr int TC_BM = 128;              // weight rows per tile (MMA M)
constexpr int TC_BN = 256;              // activation rows per tile (MMA N)
constexpr int TC_BK = 64;               // K per stage (bf16, 128 bytes)
#ifndef TC_A_STAGES_CFG
#define TC_A_STAGES_CFG 2
#endif
#ifndef TC_B_STAGES_CFG
#define TC_B_STAGES_CFG 3
#endif
constexpr int TC_A_STAGES = TC_A_STAGES_CFG;     // dequantised weight tiles (dequant warps -> MMA)
constexpr int TC_B_STAGES = TC_B_STAGES_CFG;     // activation tiles (TMA -> MMA)
// CTA-pair mode: a B stage holds half the activation rows (16 KB), so more
// stages fit; A and B stages are released together by ONE MMA commit per
// K-step (a second commit per 4 MMAs costs ~15% of the tensor pipe's rate).
#ifndef TC_PAIR_STAGES_CFG
#define TC_PAIR_STAGES_CFG 4
#endif
constexpr int TC_PAIR_A_STAGES = TC_PAIR_STAGES_CFG;
constexpr int TC_PAIR_B_STAGES = TC_PAIR_STAGES_CFG;
// Raw weight chunks (one 256-value run of blocks per row, 4 K-steps), TMA ->
// dequant warps.  The box of each type is 16-byte sized: Q4_K 144 B (a
// super-block), Q5_K 176 B, Q4_0 144 B (8 blocks of 18 B), Q8_0 272 B (8
// blocks, as 136 uint16), Q6_K 240 B (as 120 uint16) -- an aligned window
// around the 210-byte super-block, whose start within the window is
// (chunk * 210) mod 16.
template <int WT> struct TcW;
template <> struct TcW<T_Q4_K> { static constexpr int CHUNK = 144, RAW = 4, ELEM = 1; };
template <> struct TcW<T_Q5_K> { static constexpr int CHUNK = 176, RAW = 3, ELEM = 1; };
template <> struct TcW<T_Q4_0> { static constexpr int CHUNK = 144, RAW = 4, ELEM = 1; };
template <> struct TcW<T_Q6_K> { static constexpr int CHUNK = 240, RAW = 2, ELEM = 2; };
template <> struct TcW<T_Q8_0> { static constexpr int CHUNK = 272, RAW = 2, ELEM = 2; };
constexpr int TC_THREADS = 512;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;     // 16 KB
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;     // 32 KB
constexpr int TC_MAX_GROUPS = 256;
// Epilogue staging: each of the 4 epilogue warps transposes its 32-row chunk
// through shared memory so that global stores are 16-byte vectors along the
// output row.  Rows are padded to 36 words (conflict-free 128-bit reads).
constexpr int TC_STG_STRIDE = 36;
constexpr int TC_STG_BYTES = 32 * TC_STG_STRIDE * 4;   // 4608 per warp

struct TcArgs {
    int n_tiles;            // weight-row tiles per group (N/128, or F/64 in gate/up mode)
    int k;                  // reduction length (multiple of 64)
    int groups;
    const int *row_off;     // [groups + 1] activation row offsets (device)
    const int *group_w;     // optional [groups]: weight index of each group (default: g)
    int w_rows_per_group;   // weight rows of one group in the raw tensor map
    int up_offset;          // gate/up mode: row offset of the up half (F); < 0: plain mode
    int raw_chunk_bytes;    // bytes of one raw chunk box row (TcW<WT>::CHUNK)
    // epilogue
    float *out;             // plain mode: out[row * ld_out + n] (f32), or
    __nv_bfloat16 *out_bf16;//             out_bf16[row * ld_out + n]
    long long ld_out;
    const float *row_scale; // plain mode, optional: out *= row_scale[row]
    int out_t;              // plain mode, f32: store transposed, out[n * ld_out + row]
                            // (the [rows][tokens] layout of the reference's matmul)
    __nv_bfloat16 *act;     // gate/up mode: act[row * ld_act + f]
    long long ld_act;
    // plain mode, optional: expert-parallel return.  Row r of group g, in the
    // j-th run of that group (rows received from source rank s = (me + j) % G),
    // is stored as bf16 into rank s's return buffer at row ret_base[g*G + j] +
    // (r - run_off[g*G + j]), through the peer mapping, instead of into
    // out/out_bf16.
    const EpDev *ep_ret;
    // gate/up mode, optional: expert-parallel dispatch fused into the GEMM
    // (push.ep != nullptr; row_off is then the receive layout's grp_off)
    EpPush push;
    int *err;
};

__device__ __forceinline__ float silu_ref(float g)
{
    // engine/zaya.py:305: g / (1 + exp(-clip(g, -80, 80))).  The hardware
    // exponential and approximate division (a few ulp of f32) are far below
    // the bf16 rounding of the stored result, and keep the epilogue's issue
    // slots for the mainloop.
    const float c = fminf(fmaxf(g, -80.f), 80.f);
    return __fdividef(g, 1.0f + __expf(-c));
}

// ---------------------------------------------------------------- dequant
// Q4_K: one K-step (pair p of a super-block) of one tile row and one half
// (h = 0: sub-block 2p, low nibbles -> K columns 0..31; h = 1: sub-block
// 2p+1, high nibbles -> K columns 32..63) into the SWIZZLE_128B A tile.  The
// block header (d, dmin, scales) is passed in: it serves all four K-steps of
// the block and is read from shared memory once per block.
__device__ __forceinline__ void dequant_q4k_half(uint32_t raw_row, const uint4 hdr, int p, int h, uint32_t a_row,
                                                 int r)
{
    const uint4 q0 = lds128(raw_row + 16 + 32 * p), q1 = lds128(raw_row + 32 + 32 * p);
    // bytes [sc(2p), sc(2p+1), mn(2p), mn(2p+1)] (engine/dequant.py:108-113)
    const uint32_t sp = k_scales_packed(hdr, p);
    const uint32_t sc = (sp >> (8 * h)) & 0xffu, mn = (sp >> (8 * (2 + h))) & 0xffu;
    const float s = h2f(hdr.x) * (float)sc;            // exact
    const float m = h2f(hdr.x >> 16) * (float)mn;      // exact
    // q -> f = 0.5 + q/256 (byte q placed under exponent 2^-1), value = 256 s f - (128 s + m)
    const float A = 256.0f * s, B = -(128.0f * s + m);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) {                       // 16-byte chunk = 8 K columns
        uint32_t o[4];
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const uint32_t wd = w[2 * c + ww];
            const uint32_t nib = h ? ((wd >> 4) & 0x0F0F0F0Fu) : (wd & 0x0F0F0F0Fu);
            float f[4], v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) f[b] = __uint_as_float(__byte_perm(nib, 0x3F000000u, 0x7044u | (uint32_t)(b << 8)));
            ffma2(v[0], v[1], A, A, f[0], f[1], B, B);           // two values per instruction
            ffma2(v[2], v[3], A, A, f[2], f[3], B, B);
            o[2 * ww] = pack_bf16(v[0], v[1]);
            o[2 * ww + 1] = pack_bf16(v[2], v[3]);
        }
        const uint32_t chunk = (uint32_t)(4 * h + c);
        const uint32_t dst = a_row + ((chunk ^ (uint32_t)(r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3])
                     : "memory");
    }
}

// Q5_K (engine/dequant.py:122-145): as Q4_K with a fifth bit per value, bit
// g of qh[j] for value j of sub-block g; q = 0..31 still fits the f = 0.5 +
// q/256 byte trick.  Block layout: d, dmin, scales[12], qh[32], qs[128].
__device__ __forceinline__ void dequant_q5k_half(uint32_t raw_row, const uint4 hdr, int p, int h, uint32_t a_row,
                                                 int r)
{
    const uint4 q0 = lds128(raw_row + 48 + 32 * p), q1 = lds128(raw_row + 64 + 32 * p);
    const uint4 h0 = lds128(raw_row + 16), h1 = lds128(raw_row + 32);
    const uint32_t sp = k_scales_packed(hdr, p);
    const uint32_t sc = (sp >> (8 * h)) & 0xffu, mn = (sp >> (8 * (2 + h))) & 0xffu;
    const float s = h2f(hdr.x) * (float)sc;            // exact
    const float m = h2f(hdr.x >> 16) * (float)mn;      // exact
    const float A = 256.0f * s, B = -(128.0f * s + m);
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const uint32_t qh[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const int g = 2 * p + h;                            // sub-block
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t o[4];
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const uint32_t wd = w[2 * c + ww];
            const uint32_t nib = h ? ((wd >> 4) & 0x0F0F0F0Fu) : (wd & 0x0F0F0F0Fu);
            const uint32_t q = nib | (((qh[2 * c + ww] >> g) & 0x01010101u) << 4);
            float f[4], v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) f[b] = __uint_as_float(__byte_perm(q, 0x3F000000u, 0x7044u | (uint32_t)(b << 8)));
            ffma2(v[0], v[1], A, A, f[0], f[1], B, B);
            ffma2(v[2], v[3], A, A, f[2], f[3], B, B);
            o[2 * ww] = pack_bf16(v[0], v[1]);
            o[2 * ww + 1] = pack_bf16(v[2], v[3]);
        }
        const uint32_t chunk = (uint32_t)(4 * h + c);
        const uint32_t dst = a_row + ((chunk ^ (uint32_t)(r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3])
                     : "memory");
    }
}

// N consecutive 32-bit words of shared memory starting at an even address.
template <int N>
__device__ __forceinline__ void lds_run_a2(uint32_t addr, uint32_t (&w)[N])
{
    if (addr & 2u) {
        uint32_t prev = lds32(addr - 2);
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint32_t nxt = lds32(addr + 2 + 4 * i);
            w[i] = __funnelshift_r(prev, nxt, 16);
            prev = nxt;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) w[i] = lds32(addr + 4 * i);
    }
}

__device__ __forceinline__ void sts_a_chunk(uint32_t a_row, int r, int chunk, const uint32_t (&o)[4])
{
    const uint32_t dst = a_row + (((uint32_t)chunk ^ (uint32_t)(r & 7)) << 4);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(o[0]), "r"(o[1]), "r"(o[2]), "r"(o[3])
                 : "memory");
}

// Q6_K (engine/dequant.py:146-167): K-step p of the super-block at ``blk``
// (even address), half h: values 64p+32h+j = 128*hq + 32*u + j with
// hq = p/2, u = 2(p&1)+h; q = low nibble of ql[64hq+32h+j] (high nibble for
// u >= 2) | ((qh[32hq+j] >> 2u) & 3) << 4; value d * scale[8hq+2u+j/16] *
// (q - 32), exact in f32 and rounded once to bf16.
__device__ __forceinline__ void dequant_q6k_half(uint32_t blk, int p, int h, uint32_t a_row, int r)
{
    const int hq = p >> 1, u = 2 * (p & 1) + h;
    uint32_t ql[8], qh[8];
    lds_run_a2<8>(blk + 64 * hq + 32 * h, ql);
    lds_run_a2<8>(blk + 128 + 32 * hq, qh);
    const uint32_t scw = lds_u16(blk + 192 + 8 * hq + 2 * u);
    const float d = h2f(lds_u16(blk + 208));
    const float s0 = d * (float)(int)(int8_t)(scw & 0xffu), s1 = d * (float)(int)(int8_t)(scw >> 8);
    const bool hi_nib = (p & 1) != 0;
    const int sh = 2 * u;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t o[4];
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const int wi = 2 * c + ww;
            const uint32_t nib = hi_nib ? ((ql[wi] >> 4) & 0x0F0F0F0Fu) : (ql[wi] & 0x0F0F0F0Fu);
            const uint32_t q = nib | (((qh[wi] >> sh) & 0x03030303u) << 4);
            const float sc = wi < 4 ? s0 : s1;
            float f[4], v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b)       // 2^23 + q - (2^23 + 32) = q - 32, exact
                f[b] = __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7540u | (uint32_t)b));
            fsubmul2(v[0], v[1], sc, f[0], f[1], 8388640.0f);
            fsubmul2(v[2], v[3], sc, f[2], f[3], 8388640.0f);
            o[2 * ww] = pack_bf16(v[0], v[1]);
            o[2 * ww + 1] = pack_bf16(v[2], v[3]);
        }
        sts_a_chunk(a_row, r, 4 * h + c, o);
    }
}

// Q4_0 (engine/dequant.py:62-67): K-step p, half h = block 2p+h of the
// 8-block chunk (18-byte blocks at even addresses): value j < 16 = d *
// (low nibble of qs[j] - 8), j >= 16 = d * (high nibble of qs[j-16] - 8),
// exact in f32 and rounded once to bf16.
__device__ __forceinline__ void dequant_q4_0_half(uint32_t chunk, int p, int h, uint32_t a_row, int r)
{
    const uint32_t blk = chunk + 18u * (uint32_t)(2 * p + h);
    const float d = h2f(lds_u16(blk));
    uint32_t qs[4];
    lds_run_a2<4>(blk + 2, qs);
#pragma unroll
    for (int c = 0; c < 4; ++c) {                      // 8 K columns: qs[8(c&1) ..], low (c < 2) or high nibbles
        uint32_t o[4];
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const uint32_t wd = qs[2 * (c & 1) + ww];
            const uint32_t q = c < 2 ? (wd & 0x0F0F0F0Fu) : ((wd >> 4) & 0x0F0F0F0Fu);
            float f[4], v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b)       // 2^23 + q - (2^23 + 8) = q - 8, exact
                f[b] = __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7540u | (uint32_t)b));
            fsubmul2(v[0], v[1], d, f[0], f[1], 8388616.0f);
            fsubmul2(v[2], v[3], d, f[2], f[3], 8388616.0f);
            o[2 * ww] = pack_bf16(v[0], v[1]);
            o[2 * ww + 1] = pack_bf16(v[2], v[3]);
        }
        sts_a_chunk(a_row, r, 4 * h + c, o);
    }
}

// Q8_0 (engine/dequant.py:75-78): K-step p, half h = block 2p+h of the
// 8-block chunk: value d * q (int8), exact in f32, rounded once to bf16.
__device__ __forceinline__ void dequant_q8_0_half(uint32_t chunk, int p, int h, uint32_t a_row, int r)
{
    const uint32_t blk = chunk + 34u * (uint32_t)(2 * p + h);
    const float d = h2f(lds_u16(blk));
    uint32_t qs[8];
    lds_run_a2<8>(blk + 2, qs);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t o[4];
#pragma unroll
        for (int ww = 0; ww < 2; ++ww) {
            const uint32_t q = qs[2 * c + ww] ^ 0x80808080u;   // int8 + 128
            float f[4], v[4];
#pragma unroll
            for (int b = 0; b < 4; ++b)       // 2^23 + (q + 128) - (2^23 + 128) = q, exact
                f[b] = __uint_as_float(__byte_perm(q, 0x4B000000u, 0x7540u | (uint32_t)b));
            fsubmul2(v[0], v[1], d, f[0], f[1], 8388736.0f);
            fsubmul2(v[2], v[3], d, f[2], f[3], 8388736.0f);
            o[2 * ww] = pack_bf16(v[0], v[1]);
            o[2 * ww + 1] = pack_bf16(v[2], v[3]);
        }
        sts_a_chunk(a_row, r, 4 * h + c, o);
    }
}

// ---------------------------------------------------------------- fused dispatch
// The expert-parallel exchange inside the gate/up GEMM (TcArgs::push).  Warp 2
// of every CTA (idle in the plain GEMM) is a push warp; w of NW = gridDim.x.
// Every routed slot i (dispatch order, virtual expert v = d * E_loc + g owned
// by rank d) is the bf16 row h[token_of[i]], stored into rank d's receive
// buffer at row dst_off[v] + (i - offsets[v]) -- the layout the count exchange
// built (expert-major; the sources of a group in the order d, d+1, ...).
// Order: round by round of the receivers' GEMM row tiles (the count exchange
// cuts every rank's rows into tiles of EP_TILE_ROWS, group by group, and the
// tiles into rounds: a short first one, then rounds of rt tiles).  In round r each source stores, for
// every receiver d (d = me+1, me+2, ...: the ranks' stores spread over the
// receivers), its rows that fall in d's tiles [r * rt, (r+1) * rt); so the
// receivers' first tiles fill first, whatever the sizes of the experts.  The
// rows of a round are dealt round-robin over the push warps.
// The copy engine is the SM's bulk-copy unit, not the warp's registers: lane 0
// loads a row (pieces of at most TC_PUSH_ROW bytes) into one slot of a small
// shared-memory ring (1-D bulk load, completion on the slot's mbarrier) and
// stores it to the owner with a 1-D bulk store; up to TC_PUSH_NB stores are in
// flight.  After a round the warp waits for its stores to complete, fences
// (system scope) and counts itself into round_done[r]; the last one raises
// round_flag[me][r] at every rank.  A receiver's GEMM tile waits for its
// round's flag from all G sources only.
constexpr int TC_PUSH_NB = 3;          // ring slots
constexpr int TC_PUSH_ROW = 8192;      // bytes per slot (a 4096-wide bf16 row)

__device__ __forceinline__ void ep_push_rows(const EpPush &pp, int w, int NW, int lane, int *err, uint32_t ring,
                                             uint32_t bars)
{
    const EpDev *ep = pp.ep;
    const int G = ep->G, me = ep->me, El = ep->E_loc, D = ep->D;
    const uint32_t epoch = pp.epoch ? pp.epoch : ep->epoch;
    const int blocked = ep->blocked, r0t = ep->r0, rt = ep->rt, rounds = ep->rounds;
    const int n_valid = min(pp.S, __ldg(pp.offsets + G * El));   // slots past offsets[E]: bad expert ids, not sent
    const uint32_t row_bytes = 2u * (uint32_t)D;
    uint32_t k = 0;                     // transfers issued by this warp: slot k % NB, use k / NB
    bool ok = true;
    for (int r = 0; r < rounds; ++r) {
        const int q0 = ep_round_first_tile(r, r0t, rt), q1 = ep_round_first_tile(r + 1, r0t, rt);
        int acc = 0;                    // rows of this round before the current segment
        for (int dd = 1; dd <= G; ++dd) {
            const int d = (me + dd) % G;
            if ((blocked >> d) & 1) continue;
            const int *tb = ep->dtile + d * (El + 1), *gr = ep->dgrp_off + d * (El + 1);
            for (int g = 0; g < El; ++g) {
                const int t0 = tb[g], t1 = tb[g + 1];
                if (t1 <= q0 || t0 >= q1) continue;
                // d's rows of this round in group g, and my run there
                const int r0 = gr[g] + EP_TILE_ROWS * max(q0 - t0, 0);
                const int r1 = min(gr[g] + EP_TILE_ROWS * (q1 - t0), gr[g + 1]);
                const int v = d * El + g;
                const int so = min(__ldg(pp.offsets + v), n_valid);
                const int nv = min(__ldg(pp.offsets + v + 1), n_valid) - so;
                const int base = ep->dst_off[v];
                const int lo = max(r0, base), hi = min(r1, base + nv);        // rows in d's buffer
                if (hi <= lo) continue;
                const int first = lo + ((w - acc) % NW + NW) % NW;          // my rows: first, first + NW, ...
                const int cnt = hi > first ? (hi - first + NW - 1) / NW : 0;
                char *dst0 = reinterpret_cast<char *>(ep->peer_recv[d]);
                for (int jb = 0; jb < cnt && ok; jb += 32) {
                    const int tl = jb + lane < cnt ? __ldg(pp.token_of + so + (first + (jb + lane) * NW - base)) : 0;
                    const int nb = min(32, cnt - jb);
                    for (int u = 0; u < nb; ++u) {
                        const int t = __shfl_sync(0xffffffffu, tl, u);
                        if (lane != 0 || !ok) continue;
                        if (t < 0 || t >= pp.T) {
                            atomicExch(err, ERR_BAD_INDEX);
                            continue;
                        }
                        const char *src = reinterpret_cast<const char *>(pp.h) + (long long)t * row_bytes;
                        char *dst = dst0 + (long long)(first + (jb + u) * NW) * row_bytes;
                        for (uint32_t off = 0; off < row_bytes && ok; off += TC_PUSH_ROW, ++k) {
                            const uint32_t n = min((uint32_t)TC_PUSH_ROW, row_bytes - off);
                            const uint32_t slot = k % TC_PUSH_NB, bar = bars + 8u * slot;
                            const uint32_t buf = ring + slot * (uint32_t)TC_PUSH_ROW;
                            if (k >= TC_PUSH_NB) bulk_wait_read<TC_PUSH_NB - 1>();   // the slot's last store has read it
                            mbar_arrive_expect_tx(bar, n);
                            bulk_g2s(buf, src + off, n, bar);
                            if (!mbar_wait(bar, (k / TC_PUSH_NB) & 1u, err)) {
                                ok = false;
                                break;
                            }
                            bulk_s2g(dst + off, buf, n);
                            bulk_commit();
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
                }
                acc += hi - lo;
            }
        }
        if (!ok) break;                 // receivers then time out on this round and report it
        if (lane == 0) {
            bulk_wait_all();            // this round's stores have landed
            fence_proxy_async_global();
        }
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
            const unsigned old = atomicAdd(const_cast<unsigned *>(&ep->round_done[r]), 1u);
            if (old == (unsigned)NW - 1) {
                __threadfence_system();
                for (int d = 0; d < G; ++d) st_release_sys(&ep->peer_shared[d]->round_flag[me][r], epoch);
            }
        }
        __syncwarp();
    }
    if (lane == 0) bulk_wait_all();     // nothing in flight when the warp leaves
}

// ---------------------------------------------------------------- kernel
struct TileCoord {
    int g, nt, m0, rows;    // group, weight-row tile, first activation row (local), valid rows
};

__device__ __forceinline__ TileCoord tile_coord(int t, const int *tile_pref, const int *row_off, int groups,
                                                int n_tiles)
{
    int lo = 0, hi = groups;                 // largest g with tile_pref[g] <= t
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (tile_pref[mid] <= t) lo = mid; else hi = mid;
    }
    TileCoord c;
    c.g = lo;
    const int local = t - tile_pref[lo];
    const int mrows = row_off[lo + 1] - row_off[lo];
    // activation-row-tile major: the CTAs (pairs) running at the same time
    // share a few activation row tiles and one expert's weight tiles, so both
    // stay in L2 (weight-tile major made a large expert's rows, e.g. 140 MB,
    // stream from DRAM once per weight tile)
    c.m0 = (local / n_tiles) * TC_BN;
    c.nt = local % n_tiles;
    c.rows = min(TC_BN, mrows - c.m0);
    return c;
}

// PAIR = false: one CTA per tile, MMA M = 128 weight rows x N <= 256
// activation rows.  PAIR = true: a cluster of two CTAs per tile
// (tcgen05 cta_group::2), M = 256 weight rows (128 dequantised by each CTA)
// x N <= 256 activation rows (N/2 loaded by each CTA): every SM reads only
// half of the activation tile from shared memory, which halves the operand
// traffic that bounds the one-CTA form.  Barriers of the pair: the even CTA
// ("leader") owns full_a (16 dequant warps of both CTAs arrive), full_b (both
// CTAs' TMA bytes) and acc_empty (8 epilogue warps); the MMA commits arrive on
// empty_a / empty_b / acc_full in both CTAs.
// PUSH = true: the fused expert-parallel dispatch (TcArgs::push) -- one A/B
// stage fewer, which leaves room for the push warp's ring.
template <int WT, bool PAIR, bool PUSH>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                   const TcArgs a)
{
    constexpr int TC_RAW_STAGES = TcW<WT>::RAW;
    constexpr int A_ST = PAIR ? (PUSH ? TC_PAIR_A_STAGES - 1 : TC_PAIR_A_STAGES) : TC_A_STAGES;
    constexpr int B_ST = PAIR ? (PUSH ? TC_PAIR_B_STAGES - 1 : TC_PAIR_B_STAGES) : (PUSH ? TC_B_STAGES - 1 : TC_B_STAGES);
    constexpr int B_BYTES = PAIR ? TC_B_BYTES / 2 : TC_B_BYTES;       // activation rows loaded by this CTA
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-aligned base for the swizzled tiles
    const uint32_t base = (smem_addr(smem_raw) + 1023u) & ~1023u;
    const uint32_t sA = base;
    const uint32_t sB = sA + A_ST * TC_A_BYTES;
    const uint32_t sRaw = sB + B_ST * B_BYTES;
    const uint32_t raw_stage_bytes = (uint32_t)(TC_BM * a.raw_chunk_bytes);
    const uint32_t sStg = (sRaw + TC_RAW_STAGES * raw_stage_bytes + 15u) & ~15u;
    const uint32_t sPush = (sStg + 4 * TC_STG_BYTES + 127u) & ~127u;        // push ring (PUSH only)
    const uint32_t sBar = PUSH ? sPush + TC_PUSH_NB * TC_PUSH_ROW : sStg + 4 * TC_STG_BYTES;
    const uint32_t full_a = sBar;                             // [A]        dequant warps
    const uint32_t empty_a = full_a + 8 * A_ST;               // [A]        MMA commit
    const uint32_t full_b = empty_a + 8 * A_ST;               // [B]        TMA tx
    const uint32_t empty_b = full_b + 8 * B_ST;               // [B]        MMA commit
    const uint32_t raw_full = empty_b + 8 * B_ST;             // [RAW]      TMA tx
    const uint32_t raw_empty = raw_full + 8 * TC_RAW_STAGES;  // [RAW]      8 dequant warps
    const uint32_t acc_full = raw_empty + 8 * TC_RAW_STAGES;  // [2]        MMA commit
    const uint32_t acc_empty = acc_full + 16;                 // [2]        epilogue warps
    const uint32_t tmem_slot = acc_empty + 16;
    const uint32_t push_bar = tmem_slot + 8;                  // [TC_PUSH_NB] push ring loads (PUSH only)
    // the barrier that releases a B stage: its own (one CTA) or the shared A/B one (pair)
    const uint32_t empty_ab = PAIR ? empty_a : empty_b;
    static_assert(!PAIR || A_ST == B_ST, "pair mode releases A and B stages with one commit");
    static_assert(TC_BN == EP_TILE_ROWS, "the fused exchange's rounds are made of GEMM row tiles");
    __shared__ int tile_pref[TC_MAX_GROUPS + 1];
    __shared__ int row_off_s[TC_MAX_GROUPS + 1];
    __shared__ int group_w_s[TC_MAX_GROUPS];
    __shared__ int ret_run_s[EP_MAX_EXPERTS + 1];
    __shared__ int ret_base_s[EP_MAX_EXPERTS];
    __shared__ __nv_bfloat16 *ret_peer_s[EP_MAX_RANKS];
    __shared__ int ret_G;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ksteps = a.k / TC_BK;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    // the leader's copy of a barrier (cluster address); the CTA's own in one-CTA mode
    auto lead = [&](uint32_t bar) -> uint32_t { return PAIR ? mapa_shared(bar, 0) : bar; };
    // work units: tiles (one CTA) or pair tiles (two CTAs, 2 weight tiles each)
    const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int nunits = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int n_units_w = PAIR ? (a.n_tiles + 1) / 2 : a.n_tiles;    // weight-row units per group

    if (tid == 0) {
        for (int s = 0; s < A_ST; ++s) {
            mbar_init(full_a + 8 * s, PAIR ? 16 : 8);
            mbar_init(empty_a + 8 * s, 1);
        }
        for (int s = 0; s < B_ST; ++s) {
            mbar_init(full_b + 8 * s, 1);
            mbar_init(empty_b + 8 * s, 1);
        }
        for (int s = 0; s < TC_RAW_STAGES; ++s) {
            mbar_init(raw_full + 8 * s, 1);
            mbar_init(raw_empty + 8 * s, 8);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(acc_full + 8 * s, 1);
            mbar_init(acc_empty + 8 * s, PAIR ? 8 : 4);
        }
        if (PUSH)
            for (int s = 0; s < TC_PUSH_NB; ++s) mbar_init(push_bar + 8 * s, 1);
        mbar_fence_init();
    }
    // tile prefix over groups (every CTA computes the same table)
    if (warp == 2) {
        for (int g = lane; g <= a.groups; g += 32) row_off_s[g] = a.row_off[g];
        for (int g = lane; g < a.groups; g += 32) group_w_s[g] = a.group_w ? a.group_w[g] : g;
        __syncwarp();
        if (lane == 0) {
            int acc = 0;
            for (int g = 0; g < a.groups; ++g) {
                tile_pref[g] = acc;
                const int m = row_off_s[g + 1] - row_off_s[g];
                acc += (m > 0 ? (m + TC_BN - 1) / TC_BN : 0) * n_units_w;
            }
            tile_pref[a.groups] = acc;
        }
    }
    if (warp == 3 && a.ep_ret) {
        const EpDev *ep = a.ep_ret;
        const int G = ep->G, nrun = a.groups * G;
        for (int i = lane; i <= nrun; i += 32) ret_run_s[i] = ep->run_off[i];
        for (int i = lane; i < nrun; i += 32) ret_base_s[i] = ep->ret_base[i];
        if (lane < G) ret_peer_s[lane] = ep->peer_ret[(ep->me + lane) % G];     // by run position
        if (lane == 0) ret_G = G;
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, 512);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, 512);
            tmem_relinquish();
        }
        tc_fence_before();
    }
    __syncthreads();
    if (PAIR) cluster_sync_all();        // the peer's barriers are initialised before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = lds32(tmem_slot);
    const int total_tiles = tile_pref[a.groups];
    const bool gate_up = a.up_offset >= 0;
    bool ok = true;
    // this CTA's weight tile of a unit, clamped for loads (an odd tile count
    // leaves the peer of the last pair without rows: it computes a copy of the
    // leader's and stores nothing)
    auto cta_nt = [&](int nt_unit) { return PAIR ? 2 * nt_unit + (int)rank : nt_unit; };
    // activation rows per CTA in pair mode: half the tile's valid rows, rounded up to 16
    auto pair_half = [&](int rows) { return min(TC_BN / 2, (((rows + 1) >> 1) + 15) & ~15); };

    if (warp == 0) {
        // ------------------------------------------------ raw weight producer (TMA)
        if (lane == 0) {
            const int nchunks = (ksteps + 3) / 4;
            int rq = 0;
            for (int t = unit; t < total_tiles && ok; t += nunits) {
                const TileCoord c = tile_coord(t, tile_pref, row_off_s, a.groups, n_units_w);
                const int nt = min(cta_nt(c.nt), a.n_tiles - 1);
                const int wrow0 = group_w_s[c.g] * a.w_rows_per_group + (gate_up ? nt * 64 : nt * TC_BM);
                const int wrow1 = gate_up ? wrow0 + a.up_offset : wrow0 + 64;
                for (int rc = 0; rc < nchunks; ++rc, ++rq) {
                    const int rs = rq % TC_RAW_STAGES;
                    if (rq >= TC_RAW_STAGES && !mbar_wait(raw_empty + 8 * rs, ((rq / TC_RAW_STAGES) + 1) & 1, a.err)) { ok = false; break; }
                    const uint32_t dst = sRaw + rs * raw_stage_bytes;
                    mbar_arrive_expect_tx(raw_full + 8 * rs, raw_stage_bytes);
                    // box start (in map elements): 16-byte aligned, see TcW
                    const int xb = (WT == T_Q4_K || WT == T_Q4_0) ? rc * 144 : WT == T_Q5_K ? rc * 176
                                 : WT == T_Q8_0 ? rc * 136 : ((rc * 210) & ~15) >> 1;
                    tma_load_2d(dst, &map_w, xb, wrow0, raw_full + 8 * rs);
                    tma_load_2d(dst + 64 * a.raw_chunk_bytes, &map_w, xb, wrow1, raw_full + 8 * rs);
                }
            }
        }
    } else if (warp == 3) {
        // ------------------------------------------------ activation producer (TMA)
        if (lane == 0) {
            int q = 0, ready = -1;
            const EpDev *pep = PUSH ? a.push.ep : nullptr;
            const uint32_t pepoch = pep ? (a.push.epoch ? a.push.epoch : pep->epoch) : 0u;
            for (int t = unit; t < total_tiles && ok; t += nunits) {
                const TileCoord c = tile_coord(t, tile_pref, row_off_s, a.groups, n_units_w);
                if (pep) {
                    // fused dispatch: every source's rows of this tile's round have landed
                    const int rnd = ep_round_of_tile(pep->dtile[pep->me * (pep->E_loc + 1) + c.g] + c.m0 / EP_TILE_ROWS,
                                                     pep->r0, pep->rt);
                    if (rnd > ready) {
                        const EpShared *mine = pep->peer_shared[pep->me];
                        for (int s = 0; s < pep->G && ok; ++s)
                            ok = ep_wait_flag(&mine->round_flag[s][rnd], pepoch, a.err, a.push.wait_ns);
                        if (!ok) break;
                        fence_proxy_async_global();
                        ready = rnd;
                    }
                }
                const int xrow = row_off_s[c.g] + c.m0 + (PAIR ? (int)rank * pair_half(c.rows) : 0);
                for (int ks = 0; ks < ksteps; ++ks, ++q) {
                    const int s = q % B_ST;
                    if (q >= B_ST && !mbar_wait(empty_ab + 8 * s, ((q / B_ST) + 1) & 1, a.err)) { ok = false; break; }
                    if (PAIR) {
                        if (rank == 0) mbar_arrive_expect_tx(full_b + 8 * s, 2 * B_BYTES);
                        tma_load_2d_pair(sB + s * B_BYTES, &map_x, ks * TC_BK, xrow, lead(full_b + 8 * s));
                    } else {
                        mbar_arrive_expect_tx(full_b + 8 * s, B_BYTES);
                        tma_load_2d(sB + s * B_BYTES, &map_x, ks * TC_BK, xrow, full_b + 8 * s);
                    }
                }
            }
            // pair: every MMA completion signal for this CTA's stages has landed before it leaves
            if (PAIR && ok)
                for (int u = max(0, q - B_ST); u < q; ++u)
                    if (!mbar_wait(empty_ab + 8 * (u % B_ST), (u / B_ST) & 1, a.err)) break;
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (the leader's lane 0)
        if (lane == 0 && rank == 0) {
            int q = 0, acc = 0;
            for (int t = unit; t < total_tiles && ok; t += nunits, ++acc) {
                // N of this tile's MMAs: its valid activation rows rounded up to 16 (pair: 2 x half)
                const TileCoord c = tile_coord(t, tile_pref, row_off_s, a.groups, n_units_w);
                const uint32_t idesc = PAIR ? idesc_bf16(2 * TC_BM, 2 * pair_half(c.rows))
                                            : idesc_bf16(TC_BM, min(TC_BN, (c.rows + 15) & ~15));
                const int ab = acc & 1;
                if (acc >= 2 && !(PAIR ? mbar_wait_cluster(acc_empty + 8 * ab, ((acc >> 1) + 1) & 1, a.err)
                                       : mbar_wait(acc_empty + 8 * ab, ((acc >> 1) + 1) & 1, a.err))) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * TC_BN);
                for (int ks = 0; ks < ksteps; ++ks) {
                    const int sa = q % A_ST, sb = q % B_ST;
                    if (PAIR) {
                        if (!mbar_wait_cluster(full_b + 8 * sb, (q / B_ST) & 1, a.err)) { ok = false; break; }
                        if (!mbar_wait_cluster(full_a + 8 * sa, (q / A_ST) & 1, a.err)) { ok = false; break; }
                    } else {
                        if (!mbar_wait(full_b + 8 * sb, (q / B_ST) & 1, a.err)) { ok = false; break; }
                        if (!mbar_wait(full_a + 8 * sa, (q / A_ST) & 1, a.err)) { ok = false; break; }
                    }
                    tc_fence_after();
                    const uint32_t as = sA + sa * TC_A_BYTES, bs = sB + sb * B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk) {
                        if (PAIR)
                            umma_bf16_pair(d_tmem, sw128_desc(as + 32 * kk), sw128_desc(bs + 32 * kk), idesc,
                                           (ks > 0 || kk > 0) ? 1u : 0u);
                        else
                            umma_bf16(d_tmem, sw128_desc(as + 32 * kk), sw128_desc(bs + 32 * kk), idesc,
                                      (ks > 0 || kk > 0) ? 1u : 0u);
                    }
                    if (PAIR) {
                        umma_commit_pair_both(empty_a + 8 * sa);        // releases A and B stage sa == sb
                    } else {
                        umma_commit(empty_a + 8 * sa);
                        umma_commit(empty_b + 8 * sb);
                    }
                    ++q;
                }
                if (!ok) break;
                if (PAIR) umma_commit_pair_both(acc_full + 8 * ab);
                else umma_commit(acc_full + 8 * ab);
            }
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------ epilogue
        const int ew = warp - 4;
        float *stg = reinterpret_cast<float *>(smem_raw + (sStg - smem_addr(smem_raw)) + ew * TC_STG_BYTES);
        int acc = 0;
        for (int t = unit; t < total_tiles && ok; t += nunits, ++acc) {
            const TileCoord c = tile_coord(t, tile_pref, row_off_s, a.groups, n_units_w);
            const int nt = cta_nt(c.nt);
            const bool store = nt < a.n_tiles;
            const int ab = acc & 1;
            if (!mbar_wait(acc_full + 8 * ab, (acc >> 1) & 1, a.err)) { ok = false; break; }
            tc_fence_after();
            const long long row_base = row_off_s[c.g] + c.m0;
            for (int ch = 0; ch < TC_BN / 32 && store; ++ch) {
                if (ch * 32 >= c.rows) break;                       // warp-uniform
                uint32_t v[32];
                tmem_ld32(tmem_base + ((uint32_t)(32 * ew) << 16) + (uint32_t)(ab * TC_BN + 32 * ch), v);
                tmem_ld_wait();
                const int nrow = min(32, c.rows - 32 * ch);            // valid rows of this chunk
                const long long row0 = row_base + 32 * ch;
                if (gate_up) {
                    // lanes 0-15: gate of feature 16ew+l (rows j), lanes 16-31: up (rows 16+j)
                    const bool lo = lane < 16;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float mine_g = __uint_as_float(v[j]), mine_h = __uint_as_float(v[16 + j]);
                        const float recv = __shfl_xor_sync(0xffffffffu, lo ? mine_h : mine_g, 16);
                        const float gv = lo ? mine_g : recv, uv = lo ? recv : mine_h;
                        const int r = lo ? j : 16 + j;
                        stg[r * TC_STG_STRIDE + (lo ? 0 : 16) + (lane & 15)] = silu_ref(gv) * uv;
                    }
                    __syncwarp();
#pragma unroll
                    for (int it = 0; it < 2; ++it) {
                        const int r = it * 16 + (lane >> 1), part = lane & 1;
                        if (r < nrow) {
                            const float *src = stg + r * TC_STG_STRIDE + (r >= 16 ? 16 : 0) + part * 8;
                            const float4 x0 = *reinterpret_cast<const float4 *>(src);
                            const float4 x1 = *reinterpret_cast<const float4 *>(src + 4);
                            const uint4 o = make_uint4(pack_bf16(x0.x, x0.y), pack_bf16(x0.z, x0.w),
                                                       pack_bf16(x1.x, x1.y), pack_bf16(x1.z, x1.w));
                            *reinterpret_cast<uint4 *>(a.act + (row0 + r) * a.ld_act + nt * 64 + 16 * ew +
                                                       part * 8) = o;
                        }
                    }
                } else if (a.out_t) {
                    // lane = weight row n0 + lane; v[j] = activation row row0 + j: each
                    // lane stores its 32 consecutive outputs (128 contiguous bytes)
                    float *dst = a.out + (long long)(nt * TC_BM + 32 * ew + lane) * a.ld_out + row0;
                    if (nrow == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                        for (int q4 = 0; q4 < 8; ++q4)
                            reinterpret_cast<float4 *>(dst)[q4] =
                                make_float4(__uint_as_float(v[4 * q4]), __uint_as_float(v[4 * q4 + 1]),
                                            __uint_as_float(v[4 * q4 + 2]), __uint_as_float(v[4 * q4 + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nrow) dst[j] = __uint_as_float(v[j]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) stg[j * TC_STG_STRIDE + lane] = __uint_as_float(v[j]);
                    __syncwarp();
                    const int n0 = nt * TC_BM + 32 * ew;
                    if (a.out_bf16 || a.ep_ret) {
#pragma unroll
                        for (int it = 0; it < 4; ++it) {
                            const int r = it * 8 + (lane >> 2), part = lane & 3;
                            if (r < nrow) {
                                const long long row = row0 + r;
                                const float sc = a.row_scale ? __ldg(a.row_scale + row) : 1.0f;
                                const float *src = stg + r * TC_STG_STRIDE + part * 8;
                                const float4 x0 = *reinterpret_cast<const float4 *>(src);
                                const float4 x1 = *reinterpret_cast<const float4 *>(src + 4);
                                const uint4 o = make_uint4(pack_bf16(x0.x * sc, x0.y * sc),
                                                           pack_bf16(x0.z * sc, x0.w * sc),
                                                           pack_bf16(x1.x * sc, x1.y * sc),
                                                           pack_bf16(x1.z * sc, x1.w * sc));
                                __nv_bfloat16 *dst;
                                if (a.ep_ret) {
                                    const int G = ret_G;
                                    const int *run = ret_run_s + c.g * G;
                                    int s = 0;
                                    while (s + 1 < G && row >= run[s + 1]) ++s;
                                    dst = ret_peer_s[s] + (long long)(ret_base_s[c.g * G + s] + (row - run[s])) * a.ld_out;
                                } else {
                                    dst = a.out_bf16 + row * a.ld_out;
                                }
                                *reinterpret_cast<uint4 *>(dst + n0 + part * 8) = o;
                            }
                        }
                    } else {
#pragma unroll
                        for (int it = 0; it < 8; ++it) {
                            const int r = it * 4 + (lane >> 3), part = lane & 7;
                            if (r < nrow) {
                                const long long row = row0 + r;
                                const float sc = a.row_scale ? __ldg(a.row_scale + row) : 1.0f;
                                float4 x = *reinterpret_cast<const float4 *>(stg + r * TC_STG_STRIDE + part * 4);
                                x.x *= sc; x.y *= sc; x.z *= sc; x.w *= sc;
                                *reinterpret_cast<float4 *>(a.out + row * a.ld_out + n0 + part * 4) = x;
                            }
                        }
                    }
                }
                __syncwarp();                                          // staging reused by the next chunk
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (PAIR) mbar_arrive_cluster(lead(acc_empty + 8 * ab));
                else mbar_arrive(acc_empty + 8 * ab);
            }
        }
        if (a.ep_ret) __threadfence_system();        // peer stores complete before the signal
    } else if (warp == 2) {
        // ------------------------------------------------ fused dispatch (push warp)
        if (PUSH && a.push.ep) ep_push_rows(a.push, (int)blockIdx.x, (int)gridDim.x, lane, a.err, sPush, push_bar);
    } else if (warp >= 8) {
        // ------------------------------------------------ dequantisers
        const int dt = tid - 256;                   // 0..255
        const int r = dt & 127, h = dt >> 7;
        const int ew = r >> 5, l = r & 31;
        // raw row of tile row r
        const int raw_r = gate_up ? ((l < 16) ? 16 * ew + (l & 15) : 64 + 16 * ew + (l & 15)) : r;
        int q = 0, rq = 0;
        uint4 hdr = make_uint4(0, 0, 0, 0);
        for (int t = unit; t < total_tiles && ok; t += nunits) {
            for (int ks = 0; ks < ksteps && ok; ++ks) {
                const int rs = rq % TC_RAW_STAGES;
                if ((ks & 3) == 0 && !mbar_wait(raw_full + 8 * rs, (rq / TC_RAW_STAGES) & 1, a.err)) { ok = false; break; }
                const int s = q % A_ST;
                if (q >= A_ST && !mbar_wait(empty_a + 8 * s, ((q / A_ST) + 1) & 1, a.err)) { ok = false; break; }
                const uint32_t raw_row = sRaw + rs * raw_stage_bytes + (uint32_t)(raw_r * a.raw_chunk_bytes);
                const uint32_t a_row = sA + s * TC_A_BYTES + (uint32_t)(r * 128);
                if (WT == T_Q4_K) {
                    if ((ks & 3) == 0) hdr = lds128(raw_row);
                    dequant_q4k_half(raw_row, hdr, ks & 3, h, a_row, r);
                } else if (WT == T_Q5_K) {
                    if ((ks & 3) == 0) hdr = lds128(raw_row);
                    dequant_q5k_half(raw_row, hdr, ks & 3, h, a_row, r);
                } else if (WT == T_Q4_0) {
                    dequant_q4_0_half(raw_row, ks & 3, h, a_row, r);
                }
                else if (WT == T_Q6_K) dequant_q6k_half(raw_row + (uint32_t)(((ks >> 2) * 210) & 15), ks & 3, h, a_row, r);
                else dequant_q8_0_half(raw_row, ks & 3, h, a_row, r);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (PAIR) mbar_arrive_cluster(lead(full_a + 8 * s));
                    else mbar_arrive(full_a + 8 * s);
                }
                ++q;
                if ((ks & 3) == 3 || ks == ksteps - 1) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(raw_empty + 8 * rs);
                    ++rq;
                }
            }
        }
        // pair: every MMA completion signal for this CTA's A stages has landed before it leaves
        if (PAIR && ok && warp == 8 && lane == 0)
            for (int u = max(0, q - A_ST); u < q; ++u)
                if (!mbar_wait(empty_a + 8 * (u % A_ST), (u / A_ST) & 1, a.err)) break;
    }

    __syncthreads();
    if (PAIR) cluster_sync_all();        // neither CTA leaves while the other may still touch its memory
    if (warp == 1) {
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem_base, 512);
        else tmem_dealloc(tmem_base, 512);
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*PFN_encodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode()
{
    static PFN_encodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled>(p);
    });
    return fn;
}

// Raw bytes [rows, row_bytes] seen as uint16 elements, box [box_bytes x box_rows],
// no swizzle, out-of-range elements read as zero (used by the batch-1 GEMV).
cudaError_t make_map_u16_rows(CUtensorMap *m, const void *ptr, long long rows, long long row_bytes, int box_bytes,
                              int box_rows)
{
    PFN_encodeTiled enc = get_encode();
    if (!enc) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || row_bytes % 16 || box_bytes % 16 || box_bytes / 2 > 256 ||
        box_rows < 1 || box_rows > 256)
        return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 2), (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 2), (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// bf16 [rows, cols] row-major, box [64 cols x box_rows], 128-byte swizzle.
cudaError_t make_map_bf16(CUtensorMap *m, const void *ptr, long long rows, long long cols, int box_rows)
{
    PFN_encodeTiled enc = get_encode();
    if (!enc) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (cols * 2) % 16) return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// raw bytes [rows, row_bytes] seen as elements of elem_bytes (1 or 2), box
// [chunk_bytes x 64 rows], no swizzle.  Reads past the end of a row come
// back as zeros (only the Q6_K window of the last super-block reaches there).
static cudaError_t make_map_raw(CUtensorMap *m, const void *ptr, long long rows, long long row_bytes, int chunk_bytes,
                                int elem_bytes)
{
    PFN_encodeTiled enc = get_encode();
    if (!enc) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || row_bytes % 16 || chunk_bytes % 16 ||
        chunk_bytes / elem_bytes > 256)
        return cudaErrorInvalidValue;
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / elem_bytes), (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(chunk_bytes / elem_bytes), 64};
    cuuint32_t es[2] = {1, 1};
    CUresult r = enc(m, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                     const_cast<void *>(ptr), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int WT, bool PAIR, bool PUSH>
static size_t tc_gemm_smem_bytes()
{
    const int a_st = PAIR ? (PUSH ? TC_PAIR_A_STAGES - 1 : TC_PAIR_A_STAGES) : TC_A_STAGES;
    const int b_st = PAIR ? (PUSH ? TC_PAIR_B_STAGES - 1 : TC_PAIR_B_STAGES) : (PUSH ? TC_B_STAGES - 1 : TC_B_STAGES);
    return 1024 + (size_t)a_st * TC_A_BYTES + (size_t)b_st * (PAIR ? TC_B_BYTES / 2 : TC_B_BYTES) +
           (size_t)TcW<WT>::RAW * TC_BM * TcW<WT>::CHUNK + 16 + 4 * TC_STG_BYTES + 256 +
           (PUSH ? 128 + (size_t)TC_PUSH_NB * TC_PUSH_ROW + 8 * TC_PUSH_NB : 0);
}

// CTA pairs (tcgen05 cta_group::2) by default; b200q_gemm_pair_mode(0) selects
// the one-CTA form of the same kernel.
static bool g_tc_pair = true;
static int g_tc_pairs_used = 0;        // CTA pairs of the last pair-mode launch
void tc_gemm_set_pair(bool on) { g_tc_pair = on; }
int tc_gemm_pairs_used() { return g_tc_pairs_used; }

template <int WT, bool PAIR, bool PUSH>
static cudaError_t tc_launch(const CUtensorMap &mx, const CUtensorMap &mw, const TcArgs &a, int num_sms, int max_ctas,
                             cudaStream_t st)
{
    static bool attr = false;
    static int max_pairs = 0;
    const size_t smem = tc_gemm_smem_bytes<WT, PAIR, PUSH>();
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    if (PAIR) {
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
    }
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<WT, PAIR, PUSH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        if (PAIR) {
            // pairs that can be resident at once (one CTA per SM; the SMs of a pair share a GPC)
            cfg.gridDim = dim3(2 * (num_sms / 2));
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<WT, PAIR, PUSH>, &cfg);
            if (e != cudaSuccess) return e;
            max_pairs = n;
        }
        attr = true;
    }
    int units = PAIR ? std::min(num_sms / 2, max_pairs) : num_sms;
    if (max_ctas > 0) units = std::min(units, PAIR ? std::max(1, max_ctas / 2) : max_ctas);
    if (units < 1) return cudaErrorInvalidConfiguration;
    cfg.gridDim = dim3(PAIR ? 2 * units : units);
    if (PAIR) g_tc_pairs_used = units;
    return cudaLaunchKernelEx(&cfg, tc_gemm_kernel<WT, PAIR, PUSH>, mx, mw, a);
}

template <bool PUSH>
static cudaError_t tc_launch_type(int wtype, bool pair, const CUtensorMap &mx, const CUtensorMap &mw, const TcArgs &a,
                                  int num_sms, int max_ctas, cudaStream_t st)
{
    if (pair) {
        if (wtype == T_Q4_K) return tc_launch<T_Q4_K, true, PUSH>(mx, mw, a, num_sms, max_ctas, st);
        if (wtype == T_Q5_K) return tc_launch<T_Q5_K, true, PUSH>(mx, mw, a, num_sms, max_ctas, st);
        if (wtype == T_Q4_0) return tc_launch<T_Q4_0, true, PUSH>(mx, mw, a, num_sms, max_ctas, st);
        if (wtype == T_Q6_K) return tc_launch<T_Q6_K, true, PUSH>(mx, mw, a, num_sms, max_ctas, st);
        return tc_launch<T_Q8_0, true, PUSH>(mx, mw, a, num_sms, max_ctas, st);
    }
    if (wtype == T_Q4_K) return tc_launch<T_Q4_K, false, PUSH>(mx, mw, a, num_sms, max_ctas, st);
    if (wtype == T_Q5_K) return tc_launch<T_Q5_K, false, PUSH>(mx, mw, a, num_sms, max_ctas, st);
    if (wtype == T_Q4_0) return tc_launch<T_Q4_0, false, PUSH>(mx, mw, a, num_sms, max_ctas, st);
    if (wtype == T_Q6_K) return tc_launch<T_Q6_K, false, PUSH>(mx, mw, a, num_sms, max_ctas, st);
    return tc_launch<T_Q8_0, false, PUSH>(mx, mw, a, num_sms, max_ctas, st);
}

// Grouped GEMM, Q4_K / Q6_K / Q8_0 weights.
//   x        bf16 [x_rows, k] activations (rows of group g: row_off[g]..row_off[g+1])
//   w        raw GGUF blocks of groups*w_rows_per_group rows of k values each,
//            w_row_bytes apart (0: packed rows; must be a multiple of 16)
//   up_offset >= 0: gate/up mode over n_feat features (act bf16 [x_rows, ld_act]);
//            < 0: plain mode over n_feat output columns (out f32 [x_rows, ld_out]).
cudaError_t launch_tc_gemm(int wtype, const __nv_bfloat16 *x, long long x_rows, int k, const void *w,
                           long long w_row_bytes, int groups,
                               int w_rows_per_group, int up_offset, int n_feat, const int *row_off,
                               const int *group_w, int n_weight_groups, float *out, __nv_bfloat16 *out_bf16,
                               long long ld_out, const float *row_scale, __nv_bfloat16 *act, long long ld_act,
                               int *err, int num_sms, int max_ctas, cudaStream_t st, const EpDev *ep_ret,
                               bool out_t, const EpPush *push)
{
    if (k < TC_BK || k % TC_BK) return cudaErrorInvalidValue;
    // transposed output: plain f32 mode only, no row scale, no peer return
    if (out_t && (up_offset >= 0 || !out || out_bf16 || row_scale || ep_ret || ld_out < 1)) return cudaErrorInvalidValue;
    if (ep_ret && (up_offset >= 0 || groups > EP_MAX_EXPERTS)) return cudaErrorInvalidValue;
    // the epilogue stores 16-byte vectors along output rows
    if (up_offset >= 0 && ((reinterpret_cast<uintptr_t>(act) & 15) || ld_act % 8)) return cudaErrorInvalidValue;
    if (up_offset < 0 && !ep_ret && !out_t &&
        (out_bf16 ? ((reinterpret_cast<uintptr_t>(out_bf16) & 15) || ld_out % 8)
                  : ((reinterpret_cast<uintptr_t>(out) & 15) || ld_out % 4)))
        return cudaErrorInvalidValue;
    if (out_t && (reinterpret_cast<uintptr_t>(out) & 3)) return cudaErrorInvalidValue;
    if (ep_ret && ld_out % 8) return cudaErrorInvalidValue;
    // fused dispatch: gate/up mode over the receive buffer, bf16 rows of 16-byte pieces
    if (push && (up_offset < 0 || !push->ep || !push->h || !push->token_of || !push->offsets || push->S < 0 ||
                 push->T < 0 || (reinterpret_cast<uintptr_t>(push->h) & 15) || groups > EP_MAX_EXPERTS))
        return cudaErrorInvalidValue;
    if (groups < 1 || groups > TC_MAX_GROUPS || x_rows < 1) return cudaErrorInvalidValue;
    const bool gu = up_offset >= 0;
    if (gu ? (n_feat % 64) : (n_feat % TC_BM)) return cudaErrorInvalidValue;
    if (wtype != T_Q4_K && wtype != T_Q5_K && wtype != T_Q4_0 && wtype != T_Q6_K && wtype != T_Q8_0)
        return cudaErrorInvalidValue;
    if (wtype == T_Q6_K && w_row_bytes == 0 && k % 256) return cudaErrorInvalidValue;
    const int chunk = wtype == T_Q4_K ? TcW<T_Q4_K>::CHUNK : wtype == T_Q5_K ? TcW<T_Q5_K>::CHUNK
                    : wtype == T_Q4_0 ? TcW<T_Q4_0>::CHUNK : wtype == T_Q6_K ? TcW<T_Q6_K>::CHUNK
                    : TcW<T_Q8_0>::CHUNK;
    const int elem = (wtype == T_Q4_K || wtype == T_Q5_K || wtype == T_Q4_0) ? 1 : 2;
    long long row_bytes = w_row_bytes;
    if (row_bytes == 0) {
        // packed rows (Q4_K rows hold whole super-blocks: k rounded up to 256)
        row_bytes = wtype == T_Q4_K ? ((long long)k + 255) / 256 * 144
                  : wtype == T_Q5_K ? ((long long)k + 255) / 256 * 176
                  : wtype == T_Q4_0 ? ((long long)k + 31) / 32 * 18
                  : wtype == T_Q6_K ? (long long)k / 256 * 210 : (long long)k / 32 * 34;
    }
    const long long min_bytes = wtype == T_Q4_K ? ((long long)k + 255) / 256 * 144
                              : wtype == T_Q5_K ? ((long long)k + 255) / 256 * 176
                              : wtype == T_Q4_0 ? ((long long)k + 31) / 32 * 18
                              : wtype == T_Q6_K ? ((long long)k + 255) / 256 * 210 : ((long long)k + 31) / 32 * 34;
    if (row_bytes < min_bytes) return cudaErrorInvalidValue;
    CUtensorMap mx, mw;
    const bool pair = g_tc_pair;
    cudaError_t e = make_map_bf16(&mx, x, x_rows, k, pair ? TC_BN / 2 : TC_BN);
    if (e != cudaSuccess) return e;
    e = make_map_raw(&mw, w, (long long)(group_w ? n_weight_groups : groups) * w_rows_per_group, row_bytes, chunk,
                     elem);
    if (e != cudaSuccess) return e;
    TcArgs a;
    a.n_tiles = gu ? n_feat / 64 : n_feat / TC_BM;
    a.k = k;
    a.groups = groups;
    a.row_off = row_off;
    a.group_w = group_w;
    a.w_rows_per_group = w_rows_per_group;
    a.up_offset = up_offset;
    a.raw_chunk_bytes = chunk;
    a.out = out;
    a.out_bf16 = out_bf16;
    a.ld_out = ld_out;
    a.row_scale = row_scale;
    a.out_t = out_t ? 1 : 0;
    a.act = act;
    a.ld_act = ld_act;
    a.ep_ret = ep_ret;
    if (push) a.push = *push;
    else std::memset(&a.push, 0, sizeof(a.push));
    a.err = err;
    if (push) return tc_launch_type<true>(wtype, pair, mx, mw, a, num_sms, max_ctas, st);
    return tc_launch_type<false>(wtype, pair, mx, mw, a, num_sms, max_ctas, st);
}

} // namespace b200q
