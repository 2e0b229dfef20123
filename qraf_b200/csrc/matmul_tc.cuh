// matmul_tc.cuh — tensor-core path (tcgen05 + TMEM) for batches of activation
// vectors: Y[m][n] = sum_b scale[n][b] * sum_{i<32} q[n][32b+i] * X[m][32b+i],
// the reference's dispatch_matvec_q applied to M vectors
// (src/nn/backend.cpp:131-199, batched as in include/runtime/batch_scheduler.h:187-228).
//
// Arithmetic.  Each 32-element activation block is written as integers
// X = rint(x * 2^(23-e)) (2^e > max |x| of the block), split into two limbs
// X = 4096 * hi + lo with |hi|, |lo| <= 2048, which fp16 holds exactly.  Weight
// codes are fp16 too (Q8: -127..127, Q4: -8..7).  One kind::f16 MMA per
// 16-element half-block accumulates q * limb products in fp32; every product
// and partial sum is an integer below 2^24, so the per-block sums
//     D_hi[n][m][b] = sum_i q[n][i] hi[m][i],   D_lo = sum_i q[n][i] lo[m][i]
// are exact (the "per-block partial integer sums").  The epilogue forms
//     y[n][m] += fl(4096 D_hi + D_lo) * fl(scale[n][b] * 2^(e[m][b]-23))
// in fp32 on the CUDA cores, block by block.
//
// Work split.  A stage is two blocks (64 elements of K) of 128 weight rows:
// four K=16 MMAs with 128-byte-swizzled operands (two per block, each block
// into its own accumulator) and one commit, which the consumers of the stage
// (weight ring, activation ring, epilogue) wait on, a pair of stages at a time.
// A unit is 128 weight rows (the MMA's M) by 144 bytes of each
// row (8 Q4 blocks or 4 Q8 blocks; 144 keeps every copy 16-byte aligned),
// fetched by one 2-D TMA copy (the weight seen as [N][row_bytes / 4] words).
// The grid is persistent (one CTA per SM) and CTA c takes the contiguous
// units [c*U/C, (c+1)*U/C) in tile-major order ("stream-K"), so every SM gets
// the same number of weight bytes whatever the shape.  A tile covered by one
// CTA is written straight to y; a tile shared by several CTAs is summed from
// their partial results (scratch memory) by the last of them to finish, in CTA
// order, so results are deterministic.
//
// Warps (thread = weight row): 0-7 run the epilogue in two groups that split
// the vectors (warp w reads TMEM lanes 32(w%4)..+31; the hi limbs of the
// vectors sit in accumulator columns [0, MV), the lo limbs in [MV, 2 MV)), 8-11 turn the raw bytes
// of each block into fp16 codes in the MMA's shared-memory layout and pass the
// block scales on through a small ring of their own.  Warp 12 streams the raw
// weight units, warp 13 allocates TMEM and issues the MMAs, warp 14 streams
// the prepared activation tiles.  Loops keep their ring positions as counters
// (no division).  Every wait is bounded.
#pragma once

#include <cuda.h>   // CUtensorMap

#include "common.cuh"
#include "matvec_rows.cuh"   // kMaxSeg, rms_factor

namespace qraf_dev {

constexpr uint32_t kTcRows = 128;           // weight rows per tile = MMA M = TMEM lanes
constexpr uint32_t kTcUnitBytes = 144;      // raw bytes per row per unit
constexpr uint32_t kTcRawSlot = kTcRows * kTcUnitBytes;
constexpr uint32_t kTcASlot = kTcRows * 128; // one stage of fp16 codes: 128 rows x 64 elements, 128-byte swizzle
constexpr uint32_t kTcThreads = 480;
constexpr uint32_t kTcWarpXf = 8, kTcWarpRaw = 12, kTcWarpMma = 13, kTcWarpAct = 14;
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcMaxVectors = 64;      // activation vectors per launch (MMA N = 2 x 64)

struct TcParams {
    const uint8_t* w;        // [N][row_bytes], native blocks
    const uint8_t* act;      // prepared activation tiles: [nblk / 2][act_stride] bytes, each the fp16 limb
                             // tile of two blocks (n_pad * 128 bytes, 128-byte swizzle) followed by the
                             // 2 x MV block factors 2^(e - 23)
    float* y;                // [M][N]
    float* partial;          // [gridDim][2][M][128]
    uint32_t* tile_count;    // [tiles], zeroed by the prep kernel of the same call
    uint64_t row_bytes;
    uint32_t N, M, nblk;
    uint32_t n_pad;          // MMA N: 2 x (vectors rounded up to 16, 32 or 64)
    uint32_t act_stride;     // n_pad * 128 + 2 * MV * 4
    uint32_t unit_blocks;    // 8 (Q4) or 4 (Q8)
    uint32_t upt;            // units per tile = nblk / unit_blocks
    uint32_t tiles, units;
    uint32_t nraw, nab, nbb, nd, ns, nf;   // ring depths: raw units; weight, activation, accumulator, scale,
                                           // factor stages (two blocks each)
    uint32_t pdl;
    // Output fusions (tc_store).  nseg >= 2: rows [seg_row0[i], seg_row0[i+1]) are
    // weight i of a multi-weight call (weights back to back in memory, one
    // tensor map), written to seg_y[i] ([M][rows of weight i]) with bias seg_b[i];
    // nseg <= 1: y with bias seg_b[0].  accumulate: y = fl(result + y) (a
    // residual add).  Biases: fl(result + b), before the accumulation.
    uint32_t nseg, accumulate;
    float* seg_y[kMaxSeg];
    const float* seg_b[kMaxSeg];
    uint32_t seg_row0[kMaxSeg + 1];
    // Row-sharded launch (world > 0, no output fusions): as the row kernel's
    // (RowParams), rows [row_off, row_off + N) of a y with y_ld rows; every element
    // goes to this rank's y_full and, as a (call, value) word, to every peer's
    // receive array, and the CTAs then copy the other ranks' rows in
    // (sharded_gather).  call = *seq + 1, read after the dependency wait.
    float* y_full;
    uint32_t v_off;
    unsigned long long* peer_ll[kMaxWorld];
    unsigned long long* local_ll;
    uint64_t ll_cap;
    uint32_t* cta_counter;
    uint32_t* seq;
    uint32_t world, rank, y_ld, row_off;
};

// One output element of row r (of the virtual weight) and vector m of this launch.
__device__ __forceinline__ void tc_store(const TcParams& p, uint32_t r, uint32_t m, float v, uint32_t call) {
    if (p.world) {
        sharded_store(p, call, m, r, v);
        return;
    }
    float* dst;
    const float* b;
    if (p.nseg <= 1) {
        dst = p.y + static_cast<size_t>(m) * p.N + r;
        b = p.seg_b[0] ? p.seg_b[0] + r : nullptr;
    } else {
        uint32_t i = 0;
#pragma unroll
        for (int j = 1; j < kMaxSeg; ++j)
            if (static_cast<uint32_t>(j) < p.nseg && r >= p.seg_row0[j]) i = static_cast<uint32_t>(j);
        const uint32_t rr = r - p.seg_row0[i];
        dst = p.seg_y[i] + static_cast<size_t>(m) * (p.seg_row0[i + 1] - p.seg_row0[i]) + rr;
        b = p.seg_b[i] ? p.seg_b[i] + rr : nullptr;
    }
    if (b) v = __fadd_rn(v, *b);
    if (p.accumulate) v = __fadd_rn(v, *dst);
    *dst = v;
}

// ── shared-memory matrix layout: K-major, 128-byte swizzle ─────────────────
// A tile of R rows x 64 fp16 (128 bytes per row) is R/8 atoms of 1024 bytes;
// in an atom, row r's 16-byte chunk c sits at chunk position c ^ r.  The MMA
// descriptor's stride is 1024 (one atom); a K=16 step moves its start 32 bytes
// on.  Atoms must start on 1024-byte boundaries.
__device__ __forceinline__ uint32_t tc_sw128_off(uint32_t row, uint32_t chunk) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;          // leading-dimension offset (unused with K-major swizzle)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;  // stride byte offset: one 8-row atom
    d |= static_cast<uint64_t>(1u) << 46;          // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;          // 128-byte swizzle
    return d;
}

// Position of element i (0..31) of a block inside its 32 elements of K.  Q4
// codes are laid out in the order their nibbles unpack (per 8 elements:
// 0,2,4,6,1,3,5,7); the activation tiles use the same order.
template <uint32_t DT>
__device__ __forceinline__ uint32_t tc_k_slot(uint32_t i) {
    const uint32_t l = i & 7u;
    const uint32_t s = DT == kDtypeQ4 ? ((l & 1u) ? 4u + (l >> 1) : (l >> 1)) : l;
    return (i & ~7u) | s;
}

// ── tcgen05 wrappers ───────────────────────────────────────────────────────
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One tile of a 2-D tensor map (no multicast) into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// ── activation preparation: x (fp32) -> fp16 limb tiles + block factors ────
// One warp per (block b, vector slot m); lane i takes element i.  Tile rows
// m / MV+m hold hi / lo of vector m (so the accumulator columns of the hi limbs
// of consecutive vectors are adjacent, as are the lo limbs'); rows of vectors >= M are zero; each
// block pair's tile is followed by its factors (one float per block and vector
// slot).  Also
// zeroes the stream-K tile counters of the call.  A block holding a NaN or an
// infinity gets a NaN factor, so its outputs come out NaN.
//
// Block b of vector m (lane = element): the two fp16 limbs into the block
// pair's tile and the block factor 2^(e - 23) (zero for padding vectors m >= M,
// NaN for a block holding NaN or infinity).  One warp, all lanes.
template <uint32_t DT>
__device__ __forceinline__ void tc_prep_block(float v, uint32_t b, uint32_t m, uint32_t lane, uint8_t* __restrict__ act,
                                              uint32_t M, uint32_t n_pad) {
    const uint32_t half = n_pad >> 1;
    float mx = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    const bool finite = !__any_sync(0xFFFFFFFFu, !(fabsf(v) <= 3.402823466e38f));   // no NaN / inf in the block
    // 2^e > mx: e = biased exponent - 126 for normal mx (and -126 for zero / subnormal)
    const int ex = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFFu);
    const int e = (ex == 0 ? 1 : ex) - 126;
    int X = finite ? __float2int_rn(ldexpf(v, 23 - e)) : 0;
    const int hi = (X + 2048) >> 12;
    const int lo = X - hi * 4096;
    const uint32_t kk = 32u * (b & 1u) + tc_k_slot<DT>(lane);   // element of the block pair's 64
    uint8_t* tile = act + static_cast<size_t>(b >> 1) * (n_pad * 128u + 2u * half * 4u);
    *reinterpret_cast<__half*>(tile + tc_sw128_off(m, kk >> 3) + 2u * (kk & 7u)) = __int2half_rn(hi);
    *reinterpret_cast<__half*>(tile + tc_sw128_off(half + m, kk >> 3) + 2u * (kk & 7u)) = __int2half_rn(lo);
    if (lane == 0)
        reinterpret_cast<float*>(tile + n_pad * 128u)[(b & 1u) * half + m] =
            m >= M ? 0.0f : finite ? ldexpf(1.0f, e - 23) : __int_as_float(0x7FC00000);
}

template <uint32_t DT>
__global__ void __launch_bounds__(256) tc_prep_kernel(const float* __restrict__ x, uint8_t* __restrict__ act,
                                                      uint32_t* __restrict__ tile_count, uint32_t tiles, uint32_t K,
                                                      uint32_t M, uint32_t nblk, uint32_t n_pad, uint32_t pdl) {
    if (pdl) pdl_wait();
    if (pdl) pdl_launch_dependents();
    const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
    for (uint32_t i = tid; i < tiles; i += gridDim.x * blockDim.x) tile_count[i] = 0u;
    const uint32_t half = n_pad >> 1;
    const uint32_t gw = tid >> 5, lane = threadIdx.x & 31u;
    if (gw >= nblk * half) return;
    const uint32_t b = gw / half, m = gw % half;
    float v = 0.0f;
    if (m < M) v = __ldcg(x + static_cast<size_t>(m) * K + 32u * b + lane);
    tc_prep_block<DT>(v, b, m, lane, act, M, n_pad);
}

constexpr uint32_t kTcPrepBlocks = 16;   // blocks per CTA of the fused prep kernel (two per warp)

// The prep kernel with the input formed on the way (CTA (m, c) of 256 threads:
// vector slot m, blocks [16 c, 16 c + 16); RMSNorm takes the same rms_factor as
// the unfused pass, once per CTA):
// up != nullptr: the input is silu(x) * up, as swiglu_apply_kernel forms it;
// norm_w != nullptr: the input is fl(fl(x * r) * norm_w) with r = rms_factor(x),
// as rmsnorm_kernel forms it.  Results are the bits of those passes followed
// by tc_prep_kernel.
template <uint32_t DT>
__global__ void __launch_bounds__(256) tc_prep_fused_kernel(const float* __restrict__ x, const float* __restrict__ up,
                                                            const float* __restrict__ norm_w, float eps,
                                                            uint8_t* __restrict__ act, uint32_t* __restrict__ tile_count,
                                                            uint32_t tiles, uint32_t K, uint32_t M, uint32_t nblk,
                                                            uint32_t n_pad, uint32_t pdl) {
    __shared__ double red[33];
    if (pdl) pdl_wait();
    if (pdl) pdl_launch_dependents();
    const uint32_t m = blockIdx.x, lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    if (blockIdx.y == 0)
        for (uint32_t i = m * blockDim.x + threadIdx.x; i < tiles; i += gridDim.x * blockDim.x) tile_count[i] = 0u;
    const bool live = m < M;
    const float* xm = x + static_cast<size_t>(m) * K;
    const float r = (norm_w && live) ? rms_factor(xm, K, eps, red) : 1.0f;
    const uint32_t b1 = min(nblk, (blockIdx.y + 1u) * kTcPrepBlocks);
    for (uint32_t b = blockIdx.y * kTcPrepBlocks + warp; b < b1; b += blockDim.x >> 5) {
        float v = 0.0f;
        if (live) {
            v = __ldcg(xm + 32u * b + lane);
            if (up) v = (v / (1.0f + expf(-v))) * __ldcg(up + static_cast<size_t>(m) * K + 32u * b + lane);
            if (norm_w) v = __fmul_rn(__fmul_rn(v, r), norm_w[32u * b + lane]);
        }
        tc_prep_block<DT>(v, b, m, lane, act, M, n_pad);
    }
}

// ── raw block bytes -> fp16 codes in the A layout ───────────────────────────
// q: the row's 144 raw bytes of the current unit (36 words).  Writes block j's
// 32 codes (four 16-byte chunks) for row `row` into half `half` (elements
// 32 half .. 32 half + 31) of a stage's A slot and returns the block's scale.
template <uint32_t DT>
__device__ __forceinline__ float tc_transform_block(const uint32_t (&q)[36], uint32_t j, uint8_t* a_slot, uint32_t row,
                                                    uint32_t half) {
    if constexpr (DT == kDtypeQ8) {
        // block j: word 9j = fp32 scale, words 9j+1..9j+8 = codes.  Code byte c
        // (sign bit flipped) under 0x64 is the fp16 1024 + c + 128, exactly.
        const float sc = __uint_as_float(q[9 * j]);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {   // 8 codes per 16-byte chunk
            const uint32_t w0 = q[9 * j + 1 + 2 * ch] ^ 0x80808080u, w1 = q[9 * j + 2 + 2 * ch] ^ 0x80808080u;
            uint32_t h[4];
            h[0] = __byte_perm(w0, 0x64646464u, 0x4140u);
            h[1] = __byte_perm(w0, 0x64646464u, 0x4342u);
            h[2] = __byte_perm(w1, 0x64646464u, 0x4140u);
            h[3] = __byte_perm(w1, 0x64646464u, 0x4342u);
            const __half2 off = __halves2half2(__ushort_as_half(0x6480u), __ushort_as_half(0x6480u));   // 1152
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                __half2 hv = *reinterpret_cast<__half2*>(&h[k]);
                hv = __hsub2(hv, off);
                h[k] = *reinterpret_cast<uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(a_slot + tc_sw128_off(row, 4u * half + ch)) = make_uint4(h[0], h[1], h[2], h[3]);
        }
        return sc;
    } else {
        // block j at byte 18j: fp16 scale, then 16 bytes of nibbles.  For even
        // j the block starts on a word; for odd j two bytes into one.
        const uint32_t w0 = (9u * j) >> 1;   // word holding the block's first byte
        uint32_t nib[4];
        uint32_t s16;
        if ((j & 1u) == 0u) {
#pragma unroll
            for (int k = 0; k < 4; ++k) nib[k] = __funnelshift_r(q[w0 + k], q[w0 + k + 1], 16);
            s16 = q[w0] & 0xFFFFu;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) nib[k] = q[w0 + 1 + k];
            s16 = q[w0] >> 16;
        }
        const __half2 off = __halves2half2(__ushort_as_half(0x6408u), __ushort_as_half(0x6408u));   // 1032
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {   // nibble word ch = elements 8ch..8ch+7
            const uint32_t lo4 = nib[ch] & 0x0F0F0F0Fu, hi4 = (nib[ch] >> 4) & 0x0F0F0F0Fu;
            uint32_t h[4];
            h[0] = __byte_perm(lo4, 0x64646464u, 0x4140u);   // elements 0, 2
            h[1] = __byte_perm(lo4, 0x64646464u, 0x4342u);   // 4, 6
            h[2] = __byte_perm(hi4, 0x64646464u, 0x4140u);   // 1, 3
            h[3] = __byte_perm(hi4, 0x64646464u, 0x4342u);   // 5, 7
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                __half2 hv = *reinterpret_cast<__half2*>(&h[k]);
                hv = __hsub2(hv, off);
                h[k] = *reinterpret_cast<uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(a_slot + tc_sw128_off(row, 4u * half + ch)) = make_uint4(h[0], h[1], h[2], h[3]);
        }
        return half_bits_to_float(s16);
    }
}

// Wait for the whole warp: every lane polls the same phase (one warp-wide
// instruction, no divergent branch), and the vote gives every lane the same answer.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
    const bool ok = mbar_wait(bar, parity);
    return __all_sync(0xFFFFFFFFu, ok);
}

// One lane of a converged warp (the lowest); the others skip the guarded code.
__device__ __forceinline__ bool tc_elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

// Position in a ring of n slots, advanced one step at a time (no division in
// the loops): `phase` is the parity of the slot's current fill, `wrapped` says
// whether every slot has been filled once (from then on a producer waits for
// the consumer's previous phase, parity phase ^ 1).
struct Ring {
    uint32_t slot = 0, phase = 0, n;
    bool wrapped = false;
    __device__ explicit Ring(uint32_t n_) : n(n_) {}
    __device__ __forceinline__ void next() {
        if (++slot == n) {
            slot = 0;
            phase ^= 1u;
            wrapped = true;
        }
    }
};

// CTA that owns unit u (CTA c owns [floor(c U / C), floor((c+1) U / C))).
__device__ __forceinline__ uint32_t tc_owner(uint32_t u, uint32_t units, uint32_t C) {
    return static_cast<uint32_t>(((static_cast<uint64_t>(u) + 1u) * C - 1u) / units);
}
__device__ __forceinline__ uint32_t tc_start(uint32_t c, uint32_t units, uint32_t C) {
    return static_cast<uint32_t>(static_cast<uint64_t>(c) * units / C);
}

// ── the tensor-core kernel ─────────────────────────────────────────────────
// MV: activation vectors handled per launch (16, 32 or 64); n_pad = 2 MV.
// Stage st covers blocks 2st, 2st+1 of the CTA's sequence of units.  Every role
// synchronises once per PAIR of stages (2s, 2s+1): every ring depth and every
// CTA's stage count are even, so a pair sits in slots (i, i+1) of one lap of
// each ring.  Where one party arrives on a ring in stage order (the transform
// warps, the epilogue warps, tcgen05.commit), the second stage's phase implies
// the first's and only it is waited for; slots filled by separate bulk copies
// are waited for one by one.
template <uint32_t DT, uint32_t MV>
__global__ void __launch_bounds__(kTcThreads, 1) qmm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const TcParams p) {
    constexpr uint32_t UB = DT == kDtypeQ4 ? 8u : 4u;   // blocks per raw unit
    constexpr uint32_t SPU = UB / 2u;                    // stages per raw unit
    constexpr uint32_t HV = MV / 2;                      // vectors per epilogue group
    constexpr uint32_t R = 32;                           // ring of per-stage "MMA done" barriers
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand tiles (the host adds the slack)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t tile_bytes = p.n_pad * 128u;
    uint8_t* raw = smem;
    uint8_t* abuf = raw + p.nraw * kTcRawSlot;
    uint8_t* bbuf = abuf + p.nab * kTcASlot;
    float* sring = reinterpret_cast<float*>(bbuf + p.nbb * tile_bytes);   // [ns][2][128] block scales
    float* fring = sring + p.ns * 2u * kTcRows;                           // [nf][2][MV] block factors
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(fring + p.nf * 2u * MV);
    uint64_t* raw_empty = raw_full + p.nraw;
    uint64_t* a_full = raw_empty + p.nraw;
    uint64_t* b_full = a_full + p.nab;
    uint64_t* mma_done = b_full + p.nbb;        // [R], one phase per stage
    uint64_t* d_empty = mma_done + R;
    uint64_t* s_full = d_empty + p.nd;
    uint64_t* s_empty = s_full + p.ns;
    uint64_t* f_full = s_empty + p.ns;
    uint64_t* f_empty = f_full + p.nf;
    uint64_t* comb = f_empty + p.nf;            // [2]: partial results stored / decision made
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(comb + 2);
    uint32_t* bcast = tmem_slot + 1;

    if (blockDim.x != kTcThreads || p.n_pad != 2u * MV || p.M > MV || p.unit_blocks != UB || p.nab >= R ||
        p.nbb >= R || p.nd > R || 2u * p.nd * p.n_pad > kTcTmemCols ||
        ((p.nab | p.nbb | p.nd | p.ns | p.nf) & 1u) != 0u) {
        if (threadIdx.x == 0) raise_error(kErrBadLaunch);
        return;
    }
    const uint32_t C = gridDim.x, cta = blockIdx.x;
    const uint32_t u0 = tc_start(cta, p.units, C), u1 = tc_start(cta + 1, p.units, C);
    const uint32_t nunits = u1 - u0, nstages = nunits * SPU;

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < p.nraw; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], 4);    // transform warps
        }
        for (uint32_t i = 0; i < p.nab; ++i) mbar_init(&a_full[i], 4);
        for (uint32_t i = 0; i < p.nbb; ++i) mbar_init(&b_full[i], 1);
        for (uint32_t i = 0; i < R; ++i) mbar_init(&mma_done[i], 1);
        for (uint32_t i = 0; i < p.nd; ++i) mbar_init(&d_empty[i], 8);
        for (uint32_t i = 0; i < p.ns; ++i) {
            mbar_init(&s_full[i], 4);
            mbar_init(&s_empty[i], 8);
        }
        for (uint32_t i = 0; i < p.nf; ++i) {
            mbar_init(&f_full[i], 1);
            mbar_init(&f_empty[i], 8);
        }
        mbar_init(&comb[0], 8);
        mbar_init(&comb[1], 1);
        fence_mbar_init();
    }
    if (warp == kTcWarpMma) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (p.pdl) pdl_launch_dependents();

    const uint32_t k0 = u0 % p.upt, tile0 = u0 / p.upt;   // the CTA's first unit: column k0 of tile0
    if (warp == kTcWarpRaw) {
        // ── raw weight units: weights are immutable, so they stream before the dependency wait
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
            const uint64_t pol = policy_evict_first();
            Ring r(p.nraw);
            uint32_t k = k0, tile = tile0, issued = 0;
            for (uint32_t i = 0; i < nunits; ++i) {
                if (r.wrapped && !mbar_wait(&raw_empty[r.slot], r.phase ^ 1u)) break;
                mbar_arrive_expect_tx(&raw_full[r.slot], kTcRawSlot);   // rows past N arrive as zeros
                tma_load_2d(raw + r.slot * kTcRawSlot, &wmap, static_cast<int>(k * (kTcUnitBytes / 4u)),
                            static_cast<int>(tile * kTcRows), &raw_full[r.slot], pol);
                ++issued;
                r.next();
                if (++k == p.upt) {
                    k = 0;
                    ++tile;
                }
            }
            // the last unit issued into each slot has landed before the CTA leaves
            for (uint32_t i = issued > p.nraw ? issued - p.nraw : 0; i < issued; ++i)
                mbar_wait(&raw_full[i % p.nraw], (i / p.nraw) & 1u);
        }
    } else if (warp == kTcWarpAct) {
        // ── prepared activation tiles and factors (written by the prep kernel just before)
        if (lane == 0) {
            if (p.pdl) pdl_wait();
            Ring rb(p.nbb), rf(p.nf), rm(R);   // rm: the stage whose MMA frees this stage's tile slot
            uint32_t issued = 0;
            const uint8_t* src = p.act + static_cast<size_t>(k0) * SPU * p.act_stride;
            const uint8_t* row_end = p.act + static_cast<size_t>(p.upt) * SPU * p.act_stride;
            const uint32_t fbytes = 2u * MV * 4u;
            bool ok = true;
            for (uint32_t st = 0; ok && st < nstages; st += 2) {
                if (rb.wrapped) {   // the MMAs up to stage st + 1 - nbb have read both slots
                    ok = mbar_wait(&mma_done[rm.slot + 1u], rm.phase);
                    rm.next();
                    rm.next();
                    if (!ok) break;
                }
                const uint8_t* srcs[2];
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    srcs[h] = src;
                    mbar_arrive_expect_tx(&b_full[rb.slot + h], tile_bytes);
                    asm volatile(
                        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                            smem_u32(bbuf + (rb.slot + h) * tile_bytes)),
                        "l"(src), "r"(tile_bytes), "r"(smem_u32(&b_full[rb.slot + h]))
                        : "memory");
                    src += p.act_stride;
                    if (src == row_end) src = p.act;   // the next tile starts again at K = 0
                }
                if (rf.wrapped && !mbar_wait(&f_empty[rf.slot + 1u], rf.phase ^ 1u)) break;
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    mbar_arrive_expect_tx(&f_full[rf.slot + h], fbytes);
                    asm volatile(
                        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                            smem_u32(fring + (rf.slot + h) * 2u * MV)),
                        "l"(srcs[h] + tile_bytes), "r"(fbytes), "r"(smem_u32(&f_full[rf.slot + h]))
                        : "memory");
                }
                issued += 2;
                rb.next();
                rb.next();
                rf.next();
                rf.next();
            }
            for (uint32_t st = issued > p.nbb ? issued - p.nbb : 0; st < issued; ++st)
                mbar_wait(&b_full[st % p.nbb], (st / p.nbb) & 1u);
            for (uint32_t st = issued > p.nf ? issued - p.nf : 0; st < issued; ++st)
                mbar_wait(&f_full[st % p.nf], (st / p.nf) & 1u);
        }
    } else if (warp == kTcWarpMma) {
        // ── MMA issue: per stage, two K=16 MMAs per block into the block's own
        // accumulator and one commit.  The whole warp runs the loop (its operands
        // stay warp-uniform) and one elected lane issues.
        const uint32_t idesc = (1u << 4)                            // D: fp32
                               | ((p.n_pad >> 3) << 17)             // N
                               | ((kTcRows >> 4) << 24);            // M = 128; A, B: fp16, K-major
        const uint32_t a_base = smem_u32(abuf), b_base = smem_u32(bbuf);
        Ring ra(p.nab), rb(p.nbb), rd(p.nd), rm(R);
        uint32_t issued = 0, last_slot = 0, last_phase = 0;
        for (uint32_t st = 0; st < nstages; st += 2) {
            if (!warp_wait(&a_full[ra.slot + 1u], ra.phase) || !warp_wait(&b_full[rb.slot], rb.phase) ||
                !warp_wait(&b_full[rb.slot + 1u], rb.phase))
                break;
            if (rd.wrapped && !warp_wait(&d_empty[rd.slot + 1u], rd.phase ^ 1u)) break;
            tc_fence_after();
            if (tc_elect_one()) {
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t sa = a_base + (ra.slot + h) * kTcASlot, sb = b_base + (rb.slot + h) * tile_bytes;
                    const uint32_t d = tmem + (rd.slot + h) * 2u * p.n_pad;
#pragma unroll
                    for (uint32_t k = 0; k < 4; ++k)   // K = 16 steps: 32 bytes along the swizzled rows
                        tc_mma_f16(d + (k >> 1) * p.n_pad, tc_smem_desc(sa + 32u * k), tc_smem_desc(sb + 32u * k),
                                   idesc, k & 1u);
                    tc_commit(&mma_done[rm.slot + h]);
                }
            }
            __syncwarp();
            issued += 2;
            last_slot = rm.slot + 1u;
            last_phase = rm.phase;
            ra.next();
            ra.next();
            rb.next();
            rb.next();
            rd.next();
            rd.next();
            rm.next();
            rm.next();
        }
        if (issued) warp_wait(&mma_done[last_slot], last_phase);
    } else if (warp >= kTcWarpXf && warp < kTcWarpXf + 4) {
        // ── transform: raw blocks -> fp16 codes in the A ring, scales into the scale ring
        const uint32_t row = threadIdx.x - kTcWarpXf * 32u;
        uint32_t q[36];
        bool ok = true;
        Ring rr(p.nraw), ra(p.nab), rs(p.ns), rm(R);   // rm: the stage whose MMA frees this stage's A slot
        for (uint32_t i = 0; ok && i < nunits; ++i) {
            if (!warp_wait(&raw_full[rr.slot], rr.phase)) break;
            const uint4* rp = reinterpret_cast<const uint4*>(raw + rr.slot * kTcRawSlot + row * kTcUnitBytes);
#pragma unroll
            for (int k = 0; k < 9; ++k) {
                const uint4 v = rp[k];
                q[4 * k] = v.x;
                q[4 * k + 1] = v.y;
                q[4 * k + 2] = v.z;
                q[4 * k + 3] = v.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rr.slot]);
            rr.next();
#pragma unroll
            for (uint32_t j = 0; j < UB; j += 4) {   // two stages of two blocks
                if (ra.wrapped) {   // the MMAs up to stage s + 1 - nab have read both A slots
                    ok = warp_wait(&mma_done[rm.slot + 1u], rm.phase);
                    rm.next();
                    rm.next();
                }
                if (!ok || (rs.wrapped && !warp_wait(&s_empty[rs.slot + 1u], rs.phase ^ 1u))) {
                    ok = false;
                    break;
                }
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    uint8_t* a_slot = abuf + (ra.slot + h) * kTcASlot;
                    float* srow = sring + ((rs.slot + h) * 2u) * kTcRows + row;
                    srow[0] = tc_transform_block<DT>(q, j + 2u * h, a_slot, row, 0u);
                    srow[kTcRows] = tc_transform_block<DT>(q, j + 2u * h + 1u, a_slot, row, 1u);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[ra.slot]);
                    mbar_arrive(&s_full[rs.slot]);
                    mbar_arrive(&a_full[ra.slot + 1u]);
                    mbar_arrive(&s_full[rs.slot + 1u]);
                }
                ra.next();
                ra.next();
                rs.next();
                rs.next();
            }
        }
    } else if (warp < 8) {
        // ── epilogue: thread = weight row = TMEM lane; group g owns vectors [g HV, (g+1) HV)
        const uint32_t quad = warp & 3u, grp = warp >> 2;
        const uint32_t row = quad * 32u + lane;
        const uint32_t tmem_row = tmem + ((quad * 32u) << 16) + grp * HV;   // this group's hi columns; lo at +MV
        const uint32_t m0 = grp * HV;
        float acc[HV];
#pragma unroll
        for (uint32_t m = 0; m < HV; ++m) acc[m] = 0.0f;
        bool waited = false, ok = true;
        uint32_t call = 0;   // the sharded call number (world > 0), read after the dependency wait
        uint32_t ncomb = 0;
        Ring rd(p.nd), rs(p.ns), rf(p.nf), rm(R);
        uint32_t k = k0, tile = tile0;

        // one block: d[0, HV) holds the hi sums of this group's vectors, d[HV, 2 HV) the lo
        // sums.  Pairs of vectors go through the packed fp32x2 units; per element the
        // operations (and roundings) are t = fma(hi, 4096, lo), s = scale * factor,
        // acc = fma(t, s, acc).
        auto fold = [&](const uint32_t (&d)[MV], float sc, const float* pfb) {
            const float2 k4096 = make_float2(4096.0f, 4096.0f), sc2 = make_float2(sc, sc);
#pragma unroll
            for (uint32_t v = 0; v < HV; v += 2) {
                if (m0 + v < p.M) {
                    const float2 dh = make_float2(__uint_as_float(d[v]), __uint_as_float(d[v + 1]));
                    const float2 dl = make_float2(__uint_as_float(d[HV + v]), __uint_as_float(d[HV + v + 1]));
                    const float2 t = __ffma2_rn(dh, k4096, dl);
                    const float2 s2 = __fmul2_rn(sc2, *reinterpret_cast<const float2*>(pfb + m0 + v));
                    const float2 a = __ffma2_rn(t, s2, make_float2(acc[v], acc[v + 1]));
                    acc[v] = a.x;
                    acc[v + 1] = a.y;
                }
            }
        };
        auto ld8 = [&](uint32_t taddr, uint32_t* part) {
            asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                         : "=r"(part[0]), "=r"(part[1]), "=r"(part[2]), "=r"(part[3]), "=r"(part[4]), "=r"(part[5]),
                           "=r"(part[6]), "=r"(part[7])
                         : "r"(taddr));
        };
        auto ld16 = [&](uint32_t taddr, uint32_t* part) {
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(part[0]), "=r"(part[1]), "=r"(part[2]), "=r"(part[3]), "=r"(part[4]), "=r"(part[5]),
                  "=r"(part[6]), "=r"(part[7]), "=r"(part[8]), "=r"(part[9]), "=r"(part[10]), "=r"(part[11]),
                  "=r"(part[12]), "=r"(part[13]), "=r"(part[14]), "=r"(part[15])
                : "r"(taddr));
        };
        auto load_block = [&](uint32_t col, uint32_t (&d)[MV]) {
            if constexpr (HV == 8) {
                ld8(tmem_row + col, &d[0]);
                ld8(tmem_row + col + MV, &d[HV]);
            } else {
#pragma unroll
                for (uint32_t c = 0; c < HV / 16; ++c) {
                    ld16(tmem_row + col + 16u * c, &d[16 * c]);
                    ld16(tmem_row + col + MV + 16u * c, &d[HV + 16 * c]);
                }
            }
        };

        for (uint32_t iu = 0; ok && iu < nunits; ++iu) {
            const bool seg_first = iu == 0 || k == 0;
            const bool seg_last = iu + 1 == nunits || k + 1 == p.upt;
            if (seg_first) {
#pragma unroll
                for (uint32_t m = 0; m < HV; ++m) acc[m] = 0.0f;
            }
#pragma unroll 1
            for (uint32_t j = 0; j < SPU; j += 2) {   // a pair of stages
                if (!warp_wait(&mma_done[rm.slot + 1u], rm.phase) || !warp_wait(&s_full[rs.slot + 1u], rs.phase) ||
                    !warp_wait(&f_full[rf.slot], rf.phase) || !warp_wait(&f_full[rf.slot + 1u], rf.phase)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                if constexpr (MV == 16) {   // the pair's four blocks: every load, then one wait
                    uint32_t d[4][MV];
#pragma unroll
                    for (uint32_t b = 0; b < 4; ++b) load_block((rd.slot * 2u + b) * p.n_pad, d[b]);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (uint32_t b = 0; b < 4; ++b)
                        fold(d[b], sring[((rs.slot + (b >> 1)) * 2u + (b & 1u)) * kTcRows + row],
                             fring + (rf.slot + (b >> 1)) * 2u * MV + (b & 1u) * MV);
                } else {
#pragma unroll 1
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t col = (rd.slot + h) * 2u * p.n_pad;
                    const float* sc = sring + ((rs.slot + h) * 2u) * kTcRows + row;
                    const float* pf = fring + (rf.slot + h) * 2u * MV;
                    if constexpr (MV <= 32) {   // both blocks' accumulators at once
                        uint32_t d0[MV], d1[MV];
                        load_block(col, d0);
                        load_block(col + p.n_pad, d1);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        fold(d0, sc[0], pf);
                        fold(d1, sc[kTcRows], pf + MV);
                    } else {
                        uint32_t d0[MV];
                        load_block(col, d0);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        fold(d0, sc[0], pf);
                        load_block(col + p.n_pad, d0);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                        fold(d0, sc[kTcRows], pf + MV);
                    }
                }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h) {
                        mbar_arrive(&d_empty[rd.slot + h]);
                        mbar_arrive(&s_empty[rs.slot + h]);
                        mbar_arrive(&f_empty[rf.slot + h]);
                    }
                }
                rd.next();
                rd.next();
                rs.next();
                rs.next();
                rf.next();
                rf.next();
                rm.next();
                rm.next();
            }
            if (!ok) break;
            const uint32_t t_now = tile;
            if (++k == p.upt) {
                k = 0;
                ++tile;
            }
            if (!seg_last) continue;
            // ── the segment of tile t_now ends here: write it, or hand it to the combiner
            if (!waited) {
                if (p.pdl) pdl_wait();
                if (p.world) call = *reinterpret_cast<volatile const uint32_t*>(p.seq) + 1u;
                waited = true;
            }
            const uint32_t t0u = t_now * p.upt, t1u = t0u + p.upt;
            const uint32_t rows = min(kTcRows, p.N - t_now * kTcRows);
            const uint32_t grow = t_now * kTcRows + row;
            if (u0 <= t0u && u1 >= t1u) {
                if (row < rows) {
#pragma unroll
                    for (uint32_t v = 0; v < HV; ++v)
                        if (m0 + v < p.M) tc_store(p, grow, m0 + v, acc[v], call);
                }
                continue;
            }
            const uint32_t slot = t_now == tile0 ? 0u : 1u;
            float* mine = p.partial + (static_cast<size_t>(cta) * 2u + slot) * p.M * kTcRows + row;
#pragma unroll
            for (uint32_t v = 0; v < HV; ++v)
                if (m0 + v < p.M) mine[static_cast<size_t>(m0 + v) * kTcRows] = acc[v];
            __threadfence();
            __syncwarp();
            if (lane == 0) mbar_arrive(&comb[0]);
            const uint32_t c_first = tc_owner(t0u, p.units, C), c_last = tc_owner(t1u - 1u, p.units, C);
            if (threadIdx.x == 0) {
                uint32_t decision = 0;
                if (mbar_wait(&comb[0], ncomb & 1u)) {
                    const uint32_t prev = atomicAdd(p.tile_count + t_now, 1u);
                    decision = prev == c_last - c_first ? 1u : 2u;   // 1: the last one in sums the tile
                }
                *reinterpret_cast<volatile uint32_t*>(bcast) = decision;
                mbar_arrive(&comb[1]);
            }
            if (!warp_wait(&comb[1], ncomb & 1u)) break;
            ++ncomb;
            if (*reinterpret_cast<volatile uint32_t*>(bcast) != 1u) continue;
            __threadfence();
            // every vector's sum runs over the CTAs in order; one CTA's HV loads are in
            // flight together instead of one L2 round trip per (vector, CTA)
            float sum[HV];
#pragma unroll
            for (uint32_t v = 0; v < HV; ++v) sum[v] = 0.0f;
            for (uint32_t cc = c_first; cc <= c_last; ++cc) {
                const uint32_t sl = tc_start(cc, p.units, C) / p.upt == t_now ? 0u : 1u;
                const float* src = p.partial + ((static_cast<size_t>(cc) * 2u + sl) * p.M + m0) * kTcRows + row;
#pragma unroll
                for (uint32_t v = 0; v < HV; ++v)
                    if (m0 + v < p.M) sum[v] += __ldcg(src + static_cast<size_t>(v) * kTcRows);
            }
            if (row < rows) {
#pragma unroll
                for (uint32_t v = 0; v < HV; ++v)
                    if (m0 + v < p.M) tc_store(p, grow, m0 + v, sum[v], call);
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == kTcWarpMma) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
    }
    if (p.world) {   // every role is done: the other ranks' rows of this call, by all threads
        uint32_t* s_call = bcast + 1;
        if (threadIdx.x == 0) {
            if (p.pdl) pdl_wait();   // returns at once where the epilogue waited already
            *s_call = *reinterpret_cast<volatile const uint32_t*>(p.seq) + 1u;
        }
        __syncthreads();
        sharded_gather(p, *s_call);
    }
}

}  // namespace qraf_dev
