// matvec_stream.cuh — the HBM-streaming quantized matvec for block size 32.
//
// Computes y[m][n] = sum_b scale[n][b] * sum_i q[n][b][i] * x[m][32b+i] on the
// reference's native Q8_0 / Q4_0 rows (src/nn/backend.cpp:131-199 is the
// operation replaced; src/tensor/quantize.cpp:187-239 the per-row dot).
//
// Structure (one persistent CTA per SM):
//  * Each CTA owns a contiguous range of rows, i.e. a contiguous byte range of
//    the weight.  A producer warp streams it into a ring of shared-memory slots
//    with 1-D bulk copies (cp.async.bulk, completion on an mbarrier), R rows per
//    slot, all slots in flight at once.
//  * Consumer warps own a fixed 32-block "super-chunk" of K: lane l owns block
//    kc*32 + l and keeps that block's 32 activations in registers for the whole
//    kernel, so activations are read from L2 once per CTA, never per row.
//  * Per row the lane reads its block (36 B for Q8, 18 B for Q4) from shared
//    memory with 32-bit loads, turns the codes into floats with the exponent
//    magic-number method (a byte placed under the exponent of 2^23, then one
//    subtraction), and accumulates.  Two rows are processed together with the
//    packed fp32x2 instructions of sm_100a.
//  * EXACT mode reproduces the reference's operation order bit for bit:
//    block_sum = chain of fl(q*x) adds, p_b = fl(block_sum*scale), and the row
//    total is the in-order chain of fl(total + p_b).  The p_b of a row are
//    spread over lanes and warps, so they go to a per-slot buffer and the last
//    warp to finish the slot runs the chains (one row per lane).
//  * FAST mode uses fused multiply-adds and sums the per-lane products with a
//    warp-shuffle tree, then sums the super-chunk partials in a fixed order
//    (deterministic run to run).
#pragma once

#include "common.cuh"

namespace qraf_dev {

struct StreamParams {
    const uint8_t* w;        // [N][row_bytes], 16-byte aligned
    const float* x;          // [M][K], 16-byte aligned rows
    float* y;                // [M][N]
    uint64_t row_bytes;      // multiple of 16
    uint32_t N, K, M;
    uint32_t nblk;           // K / 32
    uint32_t nwk;            // warps per row = ceil(nblk / 32)
    uint32_t P;              // rows processed concurrently per CTA
    uint32_t CW;             // consumer warps = nwk * P
    uint32_t R;              // rows per slot
    uint32_t nst;            // slots in the ring
    uint32_t slot_stride;    // bytes between slots (multiple of 128)
    uint32_t pb_stride;      // bytes of partial buffer per slot
    uint32_t pb_row;         // floats per row in the partial buffer
    uint32_t rows_base;      // rows per CTA (floor)
    uint32_t rows_extra;     // the first rows_extra CTAs take one more row
};

template <int MT>
struct StreamTraits {
    static constexpr int kMaxConsumerWarps = (MT == 1) ? 16 : (MT == 2 ? 12 : 8);
    static constexpr int kMaxThreads = (kMaxConsumerWarps + 1) * 32;
};

// ── per-block arithmetic, two rows at a time ──────────────────────────────
// EXACT: fl(block_sum) chain then fl(block_sum * scale), as quantize.cpp:201-205.
// Scalar __fmul_rn / __fadd_rn on purpose: on sm_100a with CUDA 12.9, packed
// fp32x2 multiply-then-add sequences (inline add/mul.rn.f32x2 or the
// __fmul2_rn / __fadd2_rn intrinsics) came out as fused multiply-adds, measured
// against the oracle; the scalar forms are never fused.  Two rows are still
// interleaved for instruction-level parallelism.
__device__ __forceinline__ float2 q8_pair_exact(const uint32_t (&wa)[9], const uint32_t (&wb)[9], const float (&xr)[32]) {
    float acca = 0.0f, accb = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t ua = wa[1 + j] ^ 0x80808080u;
        const uint32_t ub = wb[1 + j] ^ 0x80808080u;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float qa = magic_byte(ua, t) - kMagicQ8;   // exact small integer
            const float qb = magic_byte(ub, t) - kMagicQ8;
            const float xv = xr[4 * j + t];
            acca = __fadd_rn(acca, __fmul_rn(qa, xv));
            accb = __fadd_rn(accb, __fmul_rn(qb, xv));
        }
    }
    return make_float2(__fmul_rn(acca, __uint_as_float(wa[0])), __fmul_rn(accb, __uint_as_float(wb[0])));
}

__device__ __forceinline__ float2 q8_pair_fast(const uint32_t (&wa)[9], const uint32_t (&wb)[9], const float (&xr)[32]) {
    const float2 negc = make_float2(-kMagicQ8, -kMagicQ8);
    float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t ua = wa[1 + j] ^ 0x80808080u;
        const uint32_t ub = wb[1 + j] ^ 0x80808080u;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 q = f2_add(make_float2(magic_byte(ua, t), magic_byte(ub, t)), negc);
            const float xv = xr[4 * j + t];
            if (t & 1) acc1 = f2_fma(q, make_float2(xv, xv), acc1);
            else       acc0 = f2_fma(q, make_float2(xv, xv), acc0);
        }
    }
    return f2_mul(f2_add(acc0, acc1), make_float2(__uint_as_float(wa[0]), __uint_as_float(wb[0])));
}

// Q4 element order inside a code word: byte t holds elements 2t (low nibble)
// and 2t+1 (high nibble); word j covers elements 8j .. 8j+7 (quantize.cpp:227-233).
__device__ __forceinline__ float2 q4_pair_exact(const uint32_t (&qa)[4], uint32_t sa, const uint32_t (&qb)[4], uint32_t sb,
                                                const float (&xr)[32]) {
    float acca = 0.0f, accb = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t loa = qa[j] & 0x0F0F0F0Fu, hia = (qa[j] >> 4) & 0x0F0F0F0Fu;
        const uint32_t lob = qb[j] & 0x0F0F0F0Fu, hib = (qb[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float x0 = xr[8 * j + 2 * t], x1 = xr[8 * j + 2 * t + 1];
            acca = __fadd_rn(acca, __fmul_rn(magic_byte(loa, t) - kMagicQ4, x0));
            accb = __fadd_rn(accb, __fmul_rn(magic_byte(lob, t) - kMagicQ4, x0));
            acca = __fadd_rn(acca, __fmul_rn(magic_byte(hia, t) - kMagicQ4, x1));
            accb = __fadd_rn(accb, __fmul_rn(magic_byte(hib, t) - kMagicQ4, x1));
        }
    }
    return make_float2(__fmul_rn(acca, half_bits_to_float(sa)), __fmul_rn(accb, half_bits_to_float(sb)));
}

__device__ __forceinline__ float2 q4_pair_fast(const uint32_t (&qa)[4], uint32_t sa, const uint32_t (&qb)[4], uint32_t sb,
                                               const float (&xr)[32]) {
    const float2 negc = make_float2(-kMagicQ4, -kMagicQ4);
    float2 acc0 = make_float2(0.0f, 0.0f), acc1 = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t loa = qa[j] & 0x0F0F0F0Fu, hia = (qa[j] >> 4) & 0x0F0F0F0Fu;
        const uint32_t lob = qb[j] & 0x0F0F0F0Fu, hib = (qb[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float2 q0 = f2_add(make_float2(magic_byte(loa, t), magic_byte(lob, t)), negc);
            const float2 q1 = f2_add(make_float2(magic_byte(hia, t), magic_byte(hib, t)), negc);
            const float x0 = xr[8 * j + 2 * t], x1 = xr[8 * j + 2 * t + 1];
            acc0 = f2_fma(q0, make_float2(x0, x0), acc0);
            acc1 = f2_fma(q1, make_float2(x1, x1), acc1);
        }
    }
    return f2_mul(f2_add(acc0, acc1), make_float2(half_bits_to_float(sa), half_bits_to_float(sb)));
}

// ── several activation vectors against one row (FAST, MT = 2 or 4) ───────
// xr2[p][i] holds (x[2p][i], x[2p+1][i]); acc[p] collects block sums for the
// pair of vectors; the caller scales by the block's weight scale.
template <int NP>
__device__ __forceinline__ void q8_multi_fast(const uint32_t (&wv)[9], const float2 (&xr2)[NP][32], float2 (&acc)[NP]) {
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[p] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t u = wv[1 + j] ^ 0x80808080u;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float q = magic_byte(u, t) - kMagicQ8;
#pragma unroll
            for (int p = 0; p < NP; ++p) acc[p] = f2_fma(make_float2(q, q), xr2[p][4 * j + t], acc[p]);
        }
    }
}

template <int NP>
__device__ __forceinline__ void q4_multi_fast(const uint32_t (&qw)[4], const float2 (&xr2)[NP][32], float2 (&acc)[NP]) {
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[p] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = qw[j] & 0x0F0F0F0Fu, hi = (qw[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float q0 = magic_byte(lo, t) - kMagicQ4;
            const float q1 = magic_byte(hi, t) - kMagicQ4;
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                acc[p] = f2_fma(make_float2(q0, q0), xr2[p][8 * j + 2 * t], acc[p]);
                acc[p] = f2_fma(make_float2(q1, q1), xr2[p][8 * j + 2 * t + 1], acc[p]);
            }
        }
    }
}

// Load the 32 activations of block b (zeros past K) from global memory.
__device__ __forceinline__ void load_x_block(const float* xrow, uint32_t b, uint32_t nblk, float (&xr)[32]) {
    if (b < nblk) {
        const float4* p = reinterpret_cast<const float4*>(xrow + 32u * b);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 v = __ldg(p + i);
            xr[4 * i] = v.x; xr[4 * i + 1] = v.y; xr[4 * i + 2] = v.z; xr[4 * i + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) xr[i] = 0.0f;
    }
}

// ── the kernel ────────────────────────────────────────────────────────────
template <uint32_t DT, bool EXACT, int MT>
__global__ void __launch_bounds__(StreamTraits<MT>::kMaxThreads, 1) qmv_stream_kernel(const StreamParams p) {
    static_assert(!EXACT || MT == 1, "exact mode handles one activation vector per launch");
    extern __shared__ __align__(128) uint8_t smem[];

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nst = p.nst;
    uint8_t* slots = smem;
    uint8_t* pbufs = smem + static_cast<size_t>(nst) * p.slot_stride;
    uint64_t* full = reinterpret_cast<uint64_t*>(pbufs + static_cast<size_t>(nst) * p.pb_stride);
    uint64_t* empty = full + nst;
    uint32_t* counters = reinterpret_cast<uint32_t*>(empty + nst);

    if (blockDim.x != (p.CW + 1) * 32u) {
        if (threadIdx.x == 0) raise_error(kErrBadLaunch);
        return;
    }

    // Rows of this CTA.
    const uint32_t c = blockIdx.x;
    const uint32_t r0 = c * p.rows_base + min(c, p.rows_extra);
    const uint32_t nrows = p.rows_base + (c < p.rows_extra ? 1u : 0u);
    const uint32_t nstages = (nrows + p.R - 1) / p.R;

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], p.CW);
            counters[s] = 0;
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == p.CW) {
        // ── producer ──
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            for (uint32_t s = 0; s < nstages; ++s) {
                const uint32_t slot = s % nst;
                if (s >= nst && !mbar_wait(&empty[slot], ((s / nst) - 1u) & 1u)) break;
                const uint32_t rows_s = min(p.R, nrows - s * p.R);
                const uint32_t bytes = rows_s * static_cast<uint32_t>(p.row_bytes);
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_g2s(slots + static_cast<size_t>(slot) * p.slot_stride,
                         p.w + static_cast<size_t>(r0 + s * p.R) * p.row_bytes, bytes, &full[slot], pol);
            }
        }
        return;
    }

    // ── consumers ──
    const uint32_t kc = warp % p.nwk;
    const uint32_t pslot = warp / p.nwk;
    const uint32_t b = kc * 32u + lane;
    const bool valid = b < p.nblk;
    const uint32_t bsafe = valid ? b : 0u;   // keeps shared-memory reads in the row for idle lanes

    constexpr int NP = (MT > 1) ? MT / 2 : 1;
    float xr[32];
    float2 xr2[NP][32];
    const uint32_t ngroups = (MT == 1) ? 1u : (p.M + MT - 1) / MT;

    auto load_group = [&](uint32_t g) {
        if constexpr (MT == 1) {
            load_x_block(p.x, b, p.nblk, xr);
        } else {
#pragma unroll
            for (int q = 0; q < NP; ++q) {
                float xa[32], xb[32];
                const uint32_t ma = g * MT + 2 * q, mb = ma + 1;
                if (ma < p.M) load_x_block(p.x + static_cast<size_t>(ma) * p.K, b, p.nblk, xa);
                else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) xa[i] = 0.0f;
                }
                if (mb < p.M) load_x_block(p.x + static_cast<size_t>(mb) * p.K, b, p.nblk, xb);
                else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) xb[i] = 0.0f;
                }
#pragma unroll
                for (int i = 0; i < 32; ++i) xr2[q][i] = make_float2(xa[i], xb[i]);
            }
        }
    };
    load_group(0);

    for (uint32_t s = 0; s < nstages; ++s) {
        const uint32_t slot = s % nst;
        if (!mbar_wait(&full[slot], (s / nst) & 1u)) return;
        const uint32_t rows_s = min(p.R, nrows - s * p.R);
        const uint8_t* sbase = slots + static_cast<size_t>(slot) * p.slot_stride;
        float* pb = reinterpret_cast<float*>(pbufs + static_cast<size_t>(slot) * p.pb_stride);

        if constexpr (MT == 1) {
            // Rows pslot, pslot+P, ... taken two at a time.
            for (uint32_t ra = pslot; ra < rows_s; ra += 2u * p.P) {
                const uint32_t rb_ = ra + p.P;
                const bool has_b = rb_ < rows_s;
                const uint8_t* rowa = sbase + static_cast<size_t>(ra) * p.row_bytes;
                const uint8_t* rowb = sbase + static_cast<size_t>(has_b ? rb_ : ra) * p.row_bytes;
                float2 v;
                if constexpr (DT == kDtypeQ8) {
                    uint32_t wa[9], wb[9];
                    load_q8_block(rowa, bsafe, wa);
                    load_q8_block(rowb, bsafe, wb);
                    v = EXACT ? q8_pair_exact(wa, wb, xr) : q8_pair_fast(wa, wb, xr);
                } else {
                    uint32_t qa[4], qb[4], sa, sb;
                    load_q4_block(rowa, bsafe, qa, sa);
                    load_q4_block(rowb, bsafe, qb, sb);
                    v = EXACT ? q4_pair_exact(qa, sa, qb, sb, xr) : q4_pair_fast(qa, sa, qb, sb, xr);
                }
                if constexpr (EXACT) {
                    if (valid) {
                        pb[static_cast<size_t>(ra) * p.pb_row + b] = v.x;
                        if (has_b) pb[static_cast<size_t>(rb_) * p.pb_row + b] = v.y;
                    }
                } else {
                    const float va = warp_sum(valid ? v.x : 0.0f);
                    const float vb = warp_sum(valid ? v.y : 0.0f);
                    if (lane == 0) {
                        pb[static_cast<size_t>(ra) * p.pb_row + kc] = va;
                        if (has_b) pb[static_cast<size_t>(rb_) * p.pb_row + kc] = vb;
                    }
                }
            }
        } else {
            for (uint32_t g = 0; g < ngroups; ++g) {
                if (ngroups > 1) load_group(g);
                for (uint32_t r = pslot; r < rows_s; r += p.P) {
                    const uint8_t* row = sbase + static_cast<size_t>(r) * p.row_bytes;
                    float2 acc[NP];
                    float scale;
                    if constexpr (DT == kDtypeQ8) {
                        uint32_t wv[9];
                        load_q8_block(row, bsafe, wv);
                        q8_multi_fast<NP>(wv, xr2, acc);
                        scale = __uint_as_float(wv[0]);
                    } else {
                        uint32_t qw[4], s16;
                        load_q4_block(row, bsafe, qw, s16);
                        q4_multi_fast<NP>(qw, xr2, acc);
                        scale = half_bits_to_float(s16);
                    }
#pragma unroll
                    for (int q = 0; q < NP; ++q) {
                        const float va = warp_sum(valid ? acc[q].x * scale : 0.0f);
                        const float vb = warp_sum(valid ? acc[q].y * scale : 0.0f);
                        const uint32_t ma = g * MT + 2 * q;
                        if (lane == 0) {
                            // partial layout: [row][m][kc]
                            if (ma < p.M) pb[(static_cast<size_t>(r) * p.M + ma) * p.nwk + kc] = va;
                            if (ma + 1 < p.M) pb[(static_cast<size_t>(r) * p.M + ma + 1) * p.nwk + kc] = vb;
                        }
                    }
                }
            }
        }

        // The last consumer warp to finish this slot finishes its rows.
        __syncwarp();
        uint32_t old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&counters[slot], 1u);
        }
        old = __shfl_sync(0xFFFFFFFFu, old, 0);
        if (old == p.CW - 1u) {
            __threadfence_block();
            const uint32_t row0 = r0 + s * p.R;
            for (uint32_t r = lane; r < rows_s; r += 32u) {
                if constexpr (EXACT) {
                    // total = fl(total + p_b) in block order (quantize.cpp:205).
                    const float4* q4 = reinterpret_cast<const float4*>(pb + static_cast<size_t>(r) * p.pb_row);
                    float total = 0.0f;
                    for (uint32_t i = 0; i < p.nblk / 4u; ++i) {
                        const float4 v = q4[i];
                        total = __fadd_rn(total, v.x);
                        total = __fadd_rn(total, v.y);
                        total = __fadd_rn(total, v.z);
                        total = __fadd_rn(total, v.w);
                    }
                    p.y[row0 + r] = total;
                } else if constexpr (MT == 1) {
                    const float* q = pb + static_cast<size_t>(r) * p.pb_row;
                    float t = 0.0f;
                    for (uint32_t k = 0; k < p.nwk; ++k) t += q[k];
                    p.y[row0 + r] = t;
                } else {
                    for (uint32_t m = 0; m < p.M; ++m) {
                        const float* q = pb + (static_cast<size_t>(r) * p.M + m) * p.nwk;
                        float t = 0.0f;
                        for (uint32_t k = 0; k < p.nwk; ++k) t += q[k];
                        p.y[static_cast<size_t>(m) * p.N + row0 + r] = t;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) counters[slot] = 0;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
}

}  // namespace qraf_dev
