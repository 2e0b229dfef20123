// decoder.cuh — a Llama / Qwen2 decode step on the device for M slots at once
// (continuous batching): qraf_cuda_decoder_*.  Included once, at the end of
// capi.cu, after model_store.cuh.
//
// The reference runs one request at a time: Transformer::forward_llama
// (src/nn/transformer.cpp:573-620) for one token, attention_forward and
// mlp_forward (src/nn/attention.cpp:70-183), and its BatchScheduler calls that
// forward request by request (include/runtime/batch_scheduler.h:187-228).  Here
// one step takes M slots, each with its own token, position and KV cache, and
// every projection of a layer runs once for all M rows:
//   x = embedding[token]                                         (per slot)
//   per layer:  q, k, v = RMSNorm(x) W_qkv (+ biases)            one launch
//               a = attention(RoPE(q), cache + RoPE(k), v)       one launch: RoPE,
//                                                                KV store, softmax
//               x = x + a W_o                                    one launch
//               h = silu(RMSNorm(x) W_gate) * (RMSNorm(x) W_up)  one launch
//               x = x + h W_down                                 one launch
//   logits = RMSNorm(x) W_lm_head                                one launch
// The projections are the library's (any mode: EXACT, FAST, TC, AUTO), the
// residual adds folded into their stores; every launch of a step after the
// embedding uses programmatic dependent launch, so a projection streams its
// weights while the launch before it finishes.  RoPE, softmax and SiLU use
// CUDA's powf / cosf / sinf / expf where the reference calls the C library's.
#pragma once

namespace {

constexpr uint32_t kAttnThreads = 256;
constexpr uint32_t kAttnWarps = kAttnThreads / 32u;
constexpr uint32_t kAttnMinChunk = 32;        // positions per CTA, at least (fewer CTAs for short sequences)
constexpr uint32_t kAttnMaxGroup = 16;        // query heads per KV head, at most
constexpr uint32_t kAttnMaxHeadDim = 256;
constexpr uint32_t kAttnMaxSplits = 64;       // CTAs per (slot, KV head), at most (the merge reads them all;
                                              // measured on B200, one slot at context 4096: 32 -> 64 took the
                                              // step from 2.39 to 2.27 ms, 128 was slower, 2.48)
constexpr uint32_t kAttnTile = 32;            // positions per shared-memory tile (one per lane)

// x[m] = emb[tokens[m]]; a token outside the vocabulary gives zeros and raises
// kErrBadLaunch.
__global__ void __launch_bounds__(256) dec_embed_kernel(const float* __restrict__ emb, const int32_t* __restrict__ tokens,
                                                        uint32_t vocab, uint32_t hidden, float* __restrict__ x) {
    const int32_t tok = tokens[blockIdx.x];
    const bool ok = tok >= 0 && static_cast<uint32_t>(tok) < vocab;
    if (!ok && threadIdx.x == 0) raise_error(kErrBadLaunch);
    float* xm = x + static_cast<size_t>(blockIdx.x) * hidden;
    const float* row = emb + static_cast<size_t>(ok ? tok : 0) * hidden;
    for (uint32_t i = threadIdx.x; i < hidden; i += blockDim.x) xm[i] = ok ? row[i] : 0.0f;
}

// The RoPE angles of every position (ops::rope, src/nn/ops.cpp:158-177): entry
// [pos][i / 2] = (cos val, sin val) with freq = 1 / pow(theta, i / head_dim) and
// val = pos * freq, for even i < head_dim: the expressions the reference
// evaluates on every call, evaluated once when the decoder opens.
__global__ void __launch_bounds__(256) dec_rope_table_kernel(float2* __restrict__ tab, uint32_t max_seq, uint32_t hd,
                                                             float theta) {
    const uint32_t half = hd / 2u;
    for (size_t j = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < static_cast<size_t>(max_seq) * half;
         j += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const uint32_t p = static_cast<uint32_t>(j / half), i = 2u * static_cast<uint32_t>(j % half);
        const float freq = __fdiv_rn(1.0f, powf(theta, __fdiv_rn(static_cast<float>(i), static_cast<float>(hd))));
        const float val = __fmul_rn(static_cast<float>(p), freq);
        tab[j] = make_float2(cosf(val), sinf(val));
    }
}

// (a, b) rotated by (c, s): (a c - b s, a s + b c), the reference's expressions.
__device__ __forceinline__ float2 rope_pair(float a, float b, float2 cs) {
    return make_float2(__fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y)),
                       __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x)));
}

struct AttnParams {
    const float* q;            // [M][heads * hd], before RoPE
    const float* k;            // [M][kv_dim], before RoPE
    const float* v;            // [M][kv_dim]
    const float2* rope;        // [max_seq][hd / 2]
    const int32_t* pos;        // [M]
    const int32_t* slots;      // [M]
    float* kc;                 // [max_slots][layers][max_seq][kv_dim]
    float* vc;
    float* out;                // [M][heads * hd]
    int8_t* kq;                // int8 cache (QRAF_DECODER_KV_INT8): [max_slots][layers][max_seq][kv_dim]
    int8_t* vq;
    float* ksc;                // its scales: [max_slots][layers][max_seq][kv_heads]
    float* vsc;
    float* part;               // [M][kv_heads][S][G][hd + 4]: unnormalised output, max, sum (16-byte records)
    uint32_t* counter;         // [M][kv_heads]: CTAs of the group finished (the last resets it)
    uint32_t heads, kv_heads, hd, G, layer, layers, max_seq, max_slots;
    float scale;               // 1 / sqrt(head_dim)
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Floats of dynamic shared memory: q rotated [G][hd], the new k and v [hd] each,
// two stages of K and V tiles [kAttnTile][hd + 4] each, probabilities [G][kAttnTile].
__host__ __device__ constexpr size_t attn_smem_floats(uint32_t G, uint32_t hd) {
    return static_cast<size_t>(G) * hd + 2u * hd + 4u * kAttnTile * (hd + 4u) + static_cast<size_t>(G) * kAttnTile;
}

// The int8 cache's tiles: rows of hd codes at a stride of ld8 bytes (16-byte
// aligned, an odd number of 16-byte chunks so a warp's 16-byte reads of 32 rows
// meet no bank conflict), with the rows' scales.  Bytes of dynamic shared memory:
// q rotated [G][hd] floats, the new k and v codes [hd] each, two stages of
// {K codes [T][ld8], V codes [T][ld8], K scales [T], V scales [T]}, probabilities [G][T].
__host__ __device__ constexpr uint32_t attn_ld8(uint32_t hd) { return ((hd / 16u) % 2u == 0u) ? hd + 16u : hd + 32u; }
__host__ __device__ constexpr size_t attn_stage8_bytes(uint32_t hd) {
    return 2u * kAttnTile * attn_ld8(hd) + 2u * kAttnTile * 4u;
}
__host__ __device__ constexpr size_t attn_smem_bytes8(uint32_t G, uint32_t hd) {
    return 4u * static_cast<size_t>(G) * hd + 2u * hd + 2u * attn_stage8_bytes(hd) + 4u * static_cast<size_t>(G) * kAttnTile;
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}

// QuantizedKVCache::store for one value (include/nn/kv_cache_quant.h:61-94):
// clamp(round(x * inv), -127, 127), inv = 1 / (max |x| / 127) (0 when the max is 0).
__device__ __forceinline__ int8_t kvq_code(float x, float inv) {
    return static_cast<int8_t>(fmaxf(-127.0f, fminf(127.0f, roundf(__fmul_rn(x, inv)))));
}
__device__ __forceinline__ float4 i8x4_to_f4(uint32_t w) {
    return make_float4(static_cast<float>(static_cast<int8_t>(w)), static_cast<float>(static_cast<int8_t>(w >> 8)),
                       static_cast<float>(static_cast<int8_t>(w >> 16)), static_cast<float>(static_cast<int8_t>(w >> 24)));
}

// Attention of one step, fused with RoPE and the KV-cache store
// (attention_forward, src/nn/attention.cpp:104-150).  CTA (s, kvh, m) takes slot
// m's KV head kvh and the G = heads / kv_heads query heads that share it (the
// reference's kv_h = h / kv_rep), over chunk s of positions 0 .. pos: each K and
// V row is read once for the G heads.  The chunking follows the slot's position
// on the device: chunk = ceil(seq / min(S, ceil(seq / 32))), S_eff =
// ceil(seq / chunk) <= S working CTAs, each with at least one position.  The CTA
// of the last chunk rotates the new k and stores k, v at pos in the slot's cache
// (KVCache::store, attention.cpp:39-44), and takes them from shared memory.
// A chunk goes in tiles of 32 positions, each tile's K and V rows copied to
// shared memory (cp.async, the next tile's copies in flight while this one is
// used): scores q.k_t * scale with one lane per position, the softmax running
// over the tiles (max, exp(score - max), their sum, the output rescaled when the
// max grows: the reference's softmax and weighted sum, src/nn/ops.cpp:242-259,
// attention.cpp:128-147, with 1 / sum applied once at the end).  One chunk
// writes the result; with several, each leaves a partial and the last CTA of the
// group to finish (an atomic count, no waiting) merges them:
// out = sum_c exp(max_c - max) o_c / sum_c exp(max_c - max) l_c.
// Slots of one step must be distinct.  Launched with programmatic dependent
// launch: the positions, slots and the first K/V tile (earlier steps' rows) are
// read before griddepcontrol.wait, this step's q, k and v after it.
// QPT: output quads (four dimensions of one head) per thread, ceil(G hd / 4 /
// threads).  KV8: the cache holds int8 codes with a scale per (position, KV
// head) (QRAF_DECODER_KV_INT8, the reference's QuantizedKVCache layout): scores
// are fl(dot(q, codes) * scale) * 1 / sqrt(head_dim) (dot_with_key,
// kv_cache_quant.h:113-123), and each value row's scale is folded into its
// probability.
template <uint32_t QPT, bool KV8>
__global__ void __launch_bounds__(kAttnThreads) dec_attention_kernel(const AttnParams a) {
    extern __shared__ __align__(16) float att_smem[];
    __shared__ float s_alpha[kAttnMaxGroup], s_sum[kAttnMaxGroup], s_pm[kAttnMaxSplits * kAttnMaxGroup],
        s_pl[kAttnMaxSplits * kAttnMaxGroup];
    __shared__ uint32_t s_last, s_kmax, s_vmax;
    __shared__ float s_kscale, s_vscale;
    pdl_launch_dependents();
    const uint32_t s = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const int32_t p = a.pos[m], sl = a.slots[m];
    if (!(p >= 0 && static_cast<uint32_t>(p) < a.max_seq && sl >= 0 && static_cast<uint32_t>(sl) < a.max_slots)) {
        if (tid == 0 && s == 0 && kvh == 0) raise_error(kErrBadLaunch);
        return;
    }
    const uint32_t seq = static_cast<uint32_t>(p) + 1u;
    const uint32_t s0 = min(gridDim.x, (seq + kAttnMinChunk - 1u) / kAttnMinChunk);
    const uint32_t chunk = (seq + s0 - 1u) / s0;
    const uint32_t s_eff = (seq + chunk - 1u) / chunk;
    if (s >= s_eff) return;
    const uint32_t t0 = s * chunk, t1 = min(seq, t0 + chunk);
    const uint32_t G = a.G, hd = a.hd, half = hd / 2u, kv_dim = a.kv_heads * hd, ld = hd + 4u, q4 = hd / 4u;
    float* qs = att_smem;                                  // [G][hd], rotated
    float* knew = qs + G * hd;                             // [hd]
    float* vnew = knew + hd;                               // [hd]
    float* kv_st = vnew + hd;                              // stage b: K at kv_st + 2 b T ld, V after it
    float* pr = kv_st + 4u * kAttnTile * ld;               // [G][kAttnTile]
    // the int8 layout (KV8): codes of the new row, then the two stages
    const uint32_t ld8 = attn_ld8(hd);
    int8_t* knew8 = reinterpret_cast<int8_t*>(qs + G * hd);
    int8_t* vnew8 = knew8 + hd;
    uint8_t* st8 = reinterpret_cast<uint8_t*>(vnew8 + hd);
    if constexpr (KV8) pr = reinterpret_cast<float*>(st8 + 2u * attn_stage8_bytes(hd));
    const bool owner = (s == s_eff - 1u);
    const float2* cs = a.rope + static_cast<size_t>(p) * half;
    const size_t base =
        (static_cast<size_t>(sl) * a.layers + a.layer) * a.max_seq * kv_dim + static_cast<size_t>(kvh) * hd;
    const float* kbase = a.kc + base;
    const float* vbase = a.vc + base;
    const size_t sbase = (static_cast<size_t>(sl) * a.layers + a.layer) * a.max_seq * a.kv_heads + kvh;   // scales
    auto stage8 = [&](uint32_t b, int8_t*& kc8, int8_t*& vc8, float*& kscl, float*& vscl) {
        uint8_t* st = st8 + b * attn_stage8_bytes(hd);
        kc8 = reinterpret_cast<int8_t*>(st);
        vc8 = kc8 + kAttnTile * ld8;
        kscl = reinterpret_cast<float*>(vc8 + kAttnTile * ld8);
        vscl = kscl + kAttnTile;
    };

    // tile copies: rows [tt, tt + nt) of K and V into stage b, row pos excluded
    // (it is this step's, taken from knew / vnew).  Thread: 16-byte column c0 of
    // rows r0, r0 + rstep, ... (no division in the loop)
    const uint32_t rstep = kAttnThreads / q4, c0 = tid % q4, r0 = tid / q4;
    const uint32_t q16 = hd / 16u, rstep8 = kAttnThreads / q16, c08 = tid % q16, r08 = tid / q16;
    auto issue = [&](uint32_t tt, uint32_t b) {
        const uint32_t nt = min(kAttnTile, t1 - tt);
        if constexpr (KV8) {
            int8_t *kc8, *vc8;
            float *kscl, *vscl;
            stage8(b, kc8, vc8, kscl, vscl);
            if (r08 < rstep8) {
                for (uint32_t r = r08; r < nt; r += rstep8) {
                    const uint32_t t = tt + r;
                    if (t == static_cast<uint32_t>(p)) continue;
                    const size_t off = base + static_cast<size_t>(t) * kv_dim + 16u * c08;
                    cp_async16(kc8 + r * ld8 + 16u * c08, a.kq + off);
                    cp_async16(vc8 + r * ld8 + 16u * c08, a.vq + off);
                }
            }
            if (tid < nt && tt + tid != static_cast<uint32_t>(p)) {
                cp_async4(kscl + tid, a.ksc + sbase + static_cast<size_t>(tt + tid) * a.kv_heads);
                cp_async4(vscl + tid, a.vsc + sbase + static_cast<size_t>(tt + tid) * a.kv_heads);
            }
            cp_async_commit();
            return;
        }
        float* ks = kv_st + 2u * b * kAttnTile * ld;
        float* vs = ks + kAttnTile * ld;
        if (r0 < rstep) {
            for (uint32_t r = r0; r < nt; r += rstep) {
                const uint32_t t = tt + r;
                if (t == static_cast<uint32_t>(p)) continue;
                const size_t off = static_cast<size_t>(t) * kv_dim + 4u * c0;
                cp_async16(ks + r * ld + 4u * c0, kbase + off);
                cp_async16(vs + r * ld + 4u * c0, vbase + off);
            }
        }
        cp_async_commit();
    };
    // The first tile's copies go out before the dependency wait: positions below
    // pos were written by earlier steps, and pos / slots by the caller before the
    // step, so none of it depends on the launch before this one.  q, k and v do.
    issue(t0, 0);
    pdl_wait();

    const float* qm = a.q + (static_cast<size_t>(m) * a.heads + static_cast<size_t>(kvh) * G) * hd;
    for (uint32_t j = tid; j < G * half; j += kAttnThreads) {
        const uint32_t g = j / half, i = j - g * half;
        const float2 r = rope_pair(qm[g * hd + 2u * i], qm[g * hd + 2u * i + 1u], cs[i]);
        qs[g * hd + 2u * i] = r.x;
        qs[g * hd + 2u * i + 1u] = r.y;
    }
    if (owner && KV8) {
        // the new row quantized as QuantizedKVCache::store does (kv_cache_quant.h:61-94):
        // per head scale = max |x| / 127 (NaN never the max, as std::max skips it)
        const float* km = a.k + static_cast<size_t>(m) * kv_dim + static_cast<size_t>(kvh) * hd;
        const float* vm = a.v + static_cast<size_t>(m) * kv_dim + static_cast<size_t>(kvh) * hd;
        if (tid == 0) {
            s_kmax = 0u;
            s_vmax = 0u;
        }
        __syncthreads();
        float2 kr = make_float2(0.f, 0.f);
        float vv = 0.0f;
        if (tid < half) {
            kr = rope_pair(km[2u * tid], km[2u * tid + 1u], cs[tid]);
            if (!isnan(kr.x)) atomicMax(&s_kmax, __float_as_uint(fabsf(kr.x)));
            if (!isnan(kr.y)) atomicMax(&s_kmax, __float_as_uint(fabsf(kr.y)));
        }
        if (tid < hd) {
            vv = vm[tid];
            if (!isnan(vv)) atomicMax(&s_vmax, __float_as_uint(fabsf(vv)));
        }
        __syncthreads();
        const float kscale = __fdiv_rn(__uint_as_float(s_kmax), 127.0f);
        const float vscale = __fdiv_rn(__uint_as_float(s_vmax), 127.0f);
        const float kinv = kscale > 0.0f ? __fdiv_rn(1.0f, kscale) : 0.0f;
        const float vinv = vscale > 0.0f ? __fdiv_rn(1.0f, vscale) : 0.0f;
        const size_t row = base + static_cast<size_t>(p) * kv_dim;
        if (tid < half) {
            const int8_t c0 = kvq_code(kr.x, kinv), c1 = kvq_code(kr.y, kinv);
            knew8[2u * tid] = c0;
            knew8[2u * tid + 1u] = c1;
            a.kq[row + 2u * tid] = c0;
            a.kq[row + 2u * tid + 1u] = c1;
        }
        if (tid < hd) {
            const int8_t c = kvq_code(vv, vinv);
            vnew8[tid] = c;
            a.vq[row + tid] = c;
        }
        if (tid == 0) {
            s_kscale = kscale;
            s_vscale = vscale;
            a.ksc[sbase + static_cast<size_t>(p) * a.kv_heads] = kscale;
            a.vsc[sbase + static_cast<size_t>(p) * a.kv_heads] = vscale;
        }
    }
    if (owner && !KV8) {
        const float* km = a.k + static_cast<size_t>(m) * kv_dim + static_cast<size_t>(kvh) * hd;
        const float* vm = a.v + static_cast<size_t>(m) * kv_dim + static_cast<size_t>(kvh) * hd;
        float* kdst = a.kc + base + static_cast<size_t>(p) * kv_dim;
        float* vdst = a.vc + base + static_cast<size_t>(p) * kv_dim;
        for (uint32_t i = tid; i < half; i += kAttnThreads) {
            const float2 r = rope_pair(km[2u * i], km[2u * i + 1u], cs[i]);
            knew[2u * i] = r.x;
            knew[2u * i + 1u] = r.y;
            kdst[2u * i] = r.x;
            kdst[2u * i + 1u] = r.y;
        }
        for (uint32_t d = tid; d < hd; d += kAttnThreads) {
            const float x = vm[d];
            vnew[d] = x;
            vdst[d] = x;
        }
    }

    // running softmax state: per head the max (held by the warp that scores it)
    // and the sum; the output by quads: quad j = tid + i * threads is dimensions
    // 4 (j % q4) .. +3 of head j / q4, accumulated as a float4 (four chains)
    const uint32_t nquads = G * q4;
    float4 acc[QPT];
#pragma unroll
    for (uint32_t i = 0; i < QPT; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    float run_max[kAttnMaxGroup / kAttnWarps], run_sum[kAttnMaxGroup / kAttnWarps];
#pragma unroll
    for (uint32_t i = 0; i < kAttnMaxGroup / kAttnWarps; ++i) {
        run_max[i] = -INFINITY;
        run_sum[i] = 0.0f;
    }

    __syncthreads();   // qs, knew and vnew are read across threads below
    const uint32_t ntiles = (t1 - t0 + kAttnTile - 1u) / kAttnTile;
    for (uint32_t it = 0; it < ntiles; ++it) {
        const uint32_t tt = t0 + it * kAttnTile, nt = min(kAttnTile, t1 - tt), b = it & 1u;
        if (it + 1u < ntiles) {
            issue(tt + kAttnTile, b ^ 1u);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        float* ks = kv_st + 2u * b * kAttnTile * ld;
        float* vs = ks + kAttnTile * ld;
        int8_t *kc8 = nullptr, *vc8 = nullptr;
        float *kscl = nullptr, *vscl = nullptr;
        if constexpr (KV8) stage8(b, kc8, vc8, kscl, vscl);
        if (static_cast<uint32_t>(p) >= tt && static_cast<uint32_t>(p) < tt + nt) {
            const uint32_t r = static_cast<uint32_t>(p) - tt;
            for (uint32_t j = tid; j < hd; j += kAttnThreads) {
                if constexpr (KV8) {
                    kc8[r * ld8 + j] = knew8[j];
                    vc8[r * ld8 + j] = vnew8[j];
                } else {
                    ks[r * ld + j] = knew[j];
                    vs[r * ld + j] = vnew[j];
                }
            }
            if (KV8 && tid == 0) {
                kscl[r] = s_kscale;
                vscl[r] = s_vscale;
            }
        }
        __syncthreads();
        // scores and the running softmax: warp w takes heads w, w + 8; lane = position
#pragma unroll
        for (uint32_t i = 0; i < kAttnMaxGroup / kAttnWarps; ++i) {
            const uint32_t g = warp + i * kAttnWarps;
            if (g < G) {
                float sc = -INFINITY;
                if (lane < nt) {
                    const float4* qr = reinterpret_cast<const float4*>(qs + g * hd);
                    float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;   // four chains
                    if constexpr (KV8) {
                        const uint4* kr8 = reinterpret_cast<const uint4*>(kc8 + lane * ld8);
                        for (uint32_t c = 0; c < q16; ++c) {
                            const uint4 raw = kr8[c];
                            const uint32_t wd[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                            for (uint32_t j = 0; j < 4u; ++j) {
                                const float4 kk = i8x4_to_f4(wd[j]), qq = qr[4u * c + j];
                                d0 = fmaf(qq.x, kk.x, d0);
                                d1 = fmaf(qq.y, kk.y, d1);
                                d2 = fmaf(qq.z, kk.z, d2);
                                d3 = fmaf(qq.w, kk.w, d3);
                            }
                        }
                        sc = __fmul_rn(__fmul_rn(__fadd_rn(__fadd_rn(d0, d1), __fadd_rn(d2, d3)), kscl[lane]), a.scale);
                    } else {
                        const float4* kr = reinterpret_cast<const float4*>(ks + lane * ld);
#pragma unroll 4
                        for (uint32_t c = 0; c < q4; ++c) {
                            const float4 kk = kr[c], qq = qr[c];
                            d0 = fmaf(qq.x, kk.x, d0);
                            d1 = fmaf(qq.y, kk.y, d1);
                            d2 = fmaf(qq.z, kk.z, d2);
                            d3 = fmaf(qq.w, kk.w, d3);
                        }
                        sc = __fmul_rn(__fadd_rn(__fadd_rn(d0, d1), __fadd_rn(d2, d3)), a.scale);
                    }
                }
                float mt = sc;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, o));
                const float mnew = fmaxf(run_max[i], mt);
                const float e = (lane < nt) ? expf(__fsub_rn(sc, mnew)) : 0.0f;
                if constexpr (KV8) pr[g * kAttnTile + lane] = (lane < nt) ? __fmul_rn(e, vscl[lane]) : 0.0f;
                else pr[g * kAttnTile + lane] = e;
                const float alpha = expf(__fsub_rn(run_max[i], mnew));   // 0 on the first tile
                run_sum[i] = __fadd_rn(__fmul_rn(run_sum[i], alpha), warp_sum(e));
                run_max[i] = mnew;
                if (lane == 0) s_alpha[g] = alpha;
            }
        }
        __syncthreads();
        // sum_t e_t v_t by quads: V rows as float4, probabilities four positions at a
        // time (zero past nt; the rows past nt are not read)
#pragma unroll
        for (uint32_t i = 0; i < QPT; ++i) {
            const uint32_t j = tid + i * kAttnThreads;
            if (j < nquads) {
                const uint32_t g = j / q4, c4 = 4u * (j - g * q4);
                const float al = s_alpha[g];
                float4 o = make_float4(__fmul_rn(acc[i].x, al), __fmul_rn(acc[i].y, al), __fmul_rn(acc[i].z, al),
                                       __fmul_rn(acc[i].w, al));
                const float* vcol = vs + c4;
                for (uint32_t t = 0; t < nt; t += 4u) {
                    const float4 e4 = *reinterpret_cast<const float4*>(pr + g * kAttnTile + t);
                    const float e[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
                    for (uint32_t k = 0; k < 4u; ++k) {
                        if (t + k < nt) {
                            const float4 v = KV8 ? i8x4_to_f4(*reinterpret_cast<const uint32_t*>(vc8 + (t + k) * ld8 + c4))
                                                 : *reinterpret_cast<const float4*>(vcol + (t + k) * ld);
                            o.x = fmaf(e[k], v.x, o.x);
                            o.y = fmaf(e[k], v.y, o.y);
                            o.z = fmaf(e[k], v.z, o.z);
                            o.w = fmaf(e[k], v.w, o.w);
                        }
                    }
                }
                acc[i] = o;
            }
        }
        __syncthreads();   // the stage and the probabilities are reused by the next tile
    }
#pragma unroll
    for (uint32_t i = 0; i < kAttnMaxGroup / kAttnWarps; ++i) {
        const uint32_t g = warp + i * kAttnWarps;
        if (g < G && lane == 0) {
            s_sum[g] = run_sum[i];
            s_alpha[g] = run_max[i];
        }
    }
    __syncthreads();

    float* om = a.out + (static_cast<size_t>(m) * a.heads + static_cast<size_t>(kvh) * G) * hd;
    if (s_eff == 1u) {
#pragma unroll
        for (uint32_t i = 0; i < QPT; ++i) {
            const uint32_t j = tid + i * kAttnThreads;
            if (j < nquads) {
                const uint32_t g = j / q4, c4 = 4u * (j - g * q4);
                const float inv = __fdiv_rn(1.0f, s_sum[g]);
                *reinterpret_cast<float4*>(om + g * hd + c4) =
                    make_float4(__fmul_rn(acc[i].x, inv), __fmul_rn(acc[i].y, inv), __fmul_rn(acc[i].z, inv),
                                __fmul_rn(acc[i].w, inv));
            }
        }
        return;
    }
    const size_t rec = hd + 4u;
    float* pg = a.part + ((static_cast<size_t>(m) * a.kv_heads + kvh) * gridDim.x) * G * rec;
#pragma unroll
    for (uint32_t i = 0; i < QPT; ++i) {
        const uint32_t j = tid + i * kAttnThreads;
        if (j < nquads) {
            const uint32_t g = j / q4, c4 = 4u * (j - g * q4);
            float* r = pg + (static_cast<size_t>(s) * G + g) * rec;
            *reinterpret_cast<float4*>(r + c4) = acc[i];
            if (c4 == 0) {
                r[hd] = s_alpha[g];     // the chunk's max
                r[hd + 1u] = s_sum[g];
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        uint32_t* c = a.counter + static_cast<size_t>(m) * a.kv_heads + kvh;
        s_last = (atomicAdd(c, 1u) == s_eff - 1u) ? 1u : 0u;
        if (s_last) *c = 0u;      // every CTA of the group has counted: ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // merge: the chunks' (max, sum) into shared memory, per head the overall max
    // and the chunk weights exp(max_c - max), then each output's weighted sum
    // (at most kAttnMaxSplits independent loads per output)
    for (uint32_t j = tid; j < s_eff * G; j += kAttnThreads) {
        const float* r = pg + static_cast<size_t>(j) * rec;
        s_pm[j] = __ldcg(r + hd);
        s_pl[j] = __ldcg(r + hd + 1u);
    }
    __syncthreads();
    for (uint32_t g = warp; g < G; g += kAttnWarps) {   // lane c takes chunks c, c + 32, ...
        float mx = -INFINITY;
        for (uint32_t c = lane; c < s_eff; c += 32u) mx = fmaxf(mx, s_pm[c * G + g]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
        float l = 0.0f;
        for (uint32_t c = lane; c < s_eff; c += 32u) {
            const float w = expf(__fsub_rn(s_pm[c * G + g], mx));
            l = __fadd_rn(l, __fmul_rn(w, s_pl[c * G + g]));
            s_pm[c * G + g] = w;
        }
        l = warp_sum(l);
        if (lane == 0) s_sum[g] = l;
    }
    __syncthreads();
    for (uint32_t j = tid; j < nquads; j += kAttnThreads) {   // one quad per thread, every chunk's load in flight
        const uint32_t g = j / q4, c4 = 4u * (j - g * q4);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t c0 = 0; c0 < s_eff; c0 += 8u) {   // eight chunks' loads in flight at a time
            float4 v[8];
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k)
                if (c0 + k < s_eff)
                    v[k] = __ldcg(reinterpret_cast<const float4*>(pg + (static_cast<size_t>(c0 + k) * G + g) * rec + c4));
#pragma unroll
            for (uint32_t k = 0; k < 8u; ++k) {
                if (c0 + k < s_eff) {
                    const float w = s_pm[(c0 + k) * G + g];
                    o.x = fmaf(w, v[k].x, o.x);
                    o.y = fmaf(w, v[k].y, o.y);
                    o.z = fmaf(w, v[k].z, o.z);
                    o.w = fmaf(w, v[k].w, o.w);
                }
            }
        }
        const float inv = __fdiv_rn(1.0f, s_sum[g]);
        *reinterpret_cast<float4*>(om + g * hd + c4) =
            make_float4(__fmul_rn(o.x, inv), __fmul_rn(o.y, inv), __fmul_rn(o.z, inv), __fmul_rn(o.w, inv));
    }
}

// logits[m][r] = dot(W[r], x[m]) for an F32 LM head (a tied embedding,
// dispatch_matvec_opt at transformer.cpp:607-609): one warp per (row, vector),
// lane stripes then a warp sum.
__global__ void __launch_bounds__(256) dec_f32_matvec_kernel(const float* __restrict__ w, const float* __restrict__ x,
                                                             uint32_t rows, uint32_t cols, uint32_t M,
                                                             float* __restrict__ y) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
    if (warp >= rows * M) return;
    const uint32_t m = warp / rows, r = warp - m * rows;
    const float* wr = w + static_cast<size_t>(r) * cols;
    const float* xm = x + static_cast<size_t>(m) * cols;
    float acc = 0.0f;
    for (uint32_t i = lane; i < cols; i += 32u) acc = fmaf(wr[i], xm[i], acc);
    acc = warp_sum(acc);
    if (lane == 0) y[static_cast<size_t>(m) * rows + r] = acc;
}

struct DecLayer {
    qraf_weight_t qkv[3], o, gate, up, down;
    qraf_weight_t qkv_all{}, gate_up{};   // the same bytes as one weight each (tensor-core route)
    const float* attn_norm = nullptr;
    const float* ffn_norm = nullptr;
    const float* bias[3] = {nullptr, nullptr, nullptr};
};

}  // namespace

struct qraf_decoder {
    qraf_model* model = nullptr;
    int device = 0;
    uint32_t vocab = 0, hidden = 0, layers = 0, heads = 0, kv_heads = 0, hd = 0, inter = 0, G = 1;
    uint32_t max_slots = 0, max_seq = 0;
    float theta = 10000.0f, eps = 1e-5f;
    const float* emb = nullptr;
    const float* out_norm = nullptr;
    bool tied = false;
    qraf_weight_t lm_head{};
    std::vector<DecLayer> L;
    bool kv8 = false;             // QRAF_DECODER_KV_INT8: the int8 cache below instead of kc / vc
    float* kc = nullptr;          // [max_slots][layers][max_seq][kv_dim]
    float* vc = nullptr;
    int8_t* kq = nullptr;         // [max_slots][layers][max_seq][kv_dim]
    int8_t* vq = nullptr;
    float* ksc = nullptr;         // [max_slots][layers][max_seq][kv_heads]
    float* vsc = nullptr;
    float2* rope = nullptr;       // [max_seq][hd / 2]
    float* part = nullptr;        // attention partials, sized for the largest step
    uint32_t* counter = nullptr;  // [max_slots][kv_heads]
    void (*attn_kernel)(AttnParams) = nullptr;   // the instance for this model's heads per P.V thread
    float* work = nullptr;        // x, q, k, v, attention output, h, up, normalised x (tied head)
    float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *h = nullptr, *u = nullptr,
          *xn = nullptr;
    // the tensor-core route (TC, or AUTO from three slots): every projection one
    // launch pair with its fusions; needs Q/K/V and gate/up back to back in memory
    bool tc_route = false;
};

namespace {

// CTAs per (slot, KV head) of a step of M slots: about two per SM over the
// step, at most one per 32 positions of max_seq and at most kAttnMaxSplits.
uint32_t attn_splits(const qraf_decoder* d, uint32_t M, int sm_count) {
    const uint32_t by_len = std::max<uint32_t>(1u, (d->max_seq + kAttnMinChunk - 1u) / kAttnMinChunk);
    const uint32_t groups = M * d->kv_heads;
    const uint32_t target = std::max<uint32_t>(1u, (2u * static_cast<uint32_t>(sm_count) + groups - 1u) / groups);
    return std::max<uint32_t>(1u, std::min({by_len, target, kAttnMaxSplits}));
}

}  // namespace

extern "C" {

int qraf_cuda_decoder_close(qraf_decoder_t d) {
    if (!d) return QRAF_OK;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(d->device);
    for (void* p : {static_cast<void*>(d->kq), static_cast<void*>(d->vq), static_cast<void*>(d->ksc),
                    static_cast<void*>(d->vsc)})
        if (p) cudaFree(p);
    for (void* p : {static_cast<void*>(d->kc), static_cast<void*>(d->vc), static_cast<void*>(d->rope),
                    static_cast<void*>(d->part), static_cast<void*>(d->counter), static_cast<void*>(d->work)})
        if (p) cudaFree(p);
    cudaSetDevice(cur);
    if (d->model) qraf_cuda_model_close(d->model);
    delete d;
    return QRAF_OK;
}

int qraf_cuda_decoder_open(const char* path, uint32_t max_slots, uint32_t max_seq, qraf_decoder_t* out) {
    return qraf_cuda_decoder_open_ex(path, max_slots, max_seq, 0u, out);
}

int qraf_cuda_decoder_open_ex(const char* path, uint32_t max_slots, uint32_t max_seq, uint32_t flags,
                              qraf_decoder_t* out) {
    if (!out) return fail(QRAF_ERR_INVALID, "out is NULL");
    *out = nullptr;
    if (flags & ~static_cast<uint32_t>(QRAF_DECODER_KV_INT8)) return fail(QRAF_ERR_INVALID, "unknown flags 0x%x", flags);
    if (max_slots == 0 || max_seq == 0) return fail(QRAF_ERR_INVALID, "max_slots and max_seq must be positive");
    if (max_slots > 65535u || max_seq > (1u << 24))
        return fail(QRAF_ERR_UNSUPPORTED, "max_slots above 65535 or max_seq above 2^24");
    qraf_model_t m = nullptr;
    int rc = qraf_cuda_model_open_ex(path, QRAF_MODEL_F32, &m);
    if (rc) return rc;
    std::unique_ptr<qraf_decoder> d(new qraf_decoder());
    d->model = m;
    d->device = m->device;
    auto cfg = [&](const char* key, uint32_t def) {
        auto it = m->config.find(key);
        return it == m->config.end() ? def : it->second;
    };
    auto cfgf = [&](const char* key, float def) {
        auto it = m->config.find(key);
        if (it == m->config.end()) return def;
        float f;
        std::memcpy(&f, &it->second, sizeof(f));
        return f;
    };
    auto fail_close = [&](int code, const std::string& msg) {
        qraf_cuda_decoder_close(d.release());
        return fail(code, "%s: %s", path, msg.c_str());
    };
    const auto arch = m->config_str.count("architecture") ? m->config_str["architecture"] : std::string("llama");
    if (arch != "llama" && arch != "qwen2" && arch != "mistral")
        return fail_close(QRAF_ERR_UNSUPPORTED, "architecture '" + arch + "' (the decoder runs llama / qwen2 / mistral)");
    d->vocab = cfg("vocab_size", 0);
    d->hidden = cfg("hidden_size", 0);
    d->layers = cfg("num_layers", 0);
    d->heads = cfg("num_heads", 0);
    d->kv_heads = cfg("num_kv_heads", 0);
    if (d->kv_heads == 0) d->kv_heads = d->heads;
    d->inter = cfg("intermediate_size", 0);
    d->theta = cfgf("rope_theta", 10000.0f);
    d->eps = cfgf("rms_norm_eps", 1e-5f);
    if (!d->vocab || !d->hidden || !d->layers || !d->heads || !d->inter || d->hidden % d->heads ||
        d->heads % d->kv_heads)
        return fail_close(QRAF_ERR_INVALID,
                          "config lacks vocab / hidden / layers / heads / intermediate sizes or has inconsistent heads");
    d->hd = d->hidden / d->heads;
    d->G = d->heads / d->kv_heads;
    if (d->hd % 8u || d->hd > kAttnMaxHeadDim)
        return fail_close(QRAF_ERR_UNSUPPORTED, "head_dim must be a multiple of 8, at most 256");
    if (d->G > kAttnMaxGroup) return fail_close(QRAF_ERR_UNSUPPORTED, "more than 16 query heads per KV head");
    if (d->hidden % 8u) return fail_close(QRAF_ERR_UNSUPPORTED, "hidden_size must be a multiple of 8");
    d->max_slots = max_slots;
    d->max_seq = max_seq;
    auto f32 = [&](const std::string& name, uint64_t count, const float** outp, bool required) -> bool {
        auto it = m->f32.find(name);
        if (it == m->f32.end() || it->second.second != count) {
            if (required)
                fail(QRAF_ERR_INVALID, "%s: F32 tensor '%s' of %llu elements missing", path, name.c_str(),
                     static_cast<unsigned long long>(count));
            *outp = nullptr;
            return !required;
        }
        *outp = it->second.first;
        return true;
    };
    auto qw = [&](const std::string& name, uint32_t rows, uint32_t cols, qraf_weight_t* w) -> bool {
        auto it = m->weights.find(name);
        if (it == m->weights.end() || it->second.rows != rows || it->second.cols != cols) {
            fail(QRAF_ERR_INVALID, "%s: quantized tensor '%s' [%u][%u] missing", path, name.c_str(), rows, cols);
            return false;
        }
        *w = it->second;
        return true;
    };
    const uint32_t q_dim = d->heads * d->hd, kv_dim = d->kv_heads * d->hd;
    bool ok = f32("model.embed_tokens.weight", static_cast<uint64_t>(d->vocab) * d->hidden, &d->emb, true) &&
              f32("model.norm.weight", d->hidden, &d->out_norm, true);
    d->L.resize(d->layers);
    for (uint32_t l = 0; ok && l < d->layers; ++l) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        DecLayer& ly = d->L[l];
        ok = qw(p + "self_attn.q_proj.weight", q_dim, d->hidden, &ly.qkv[0]) &&
             qw(p + "self_attn.k_proj.weight", kv_dim, d->hidden, &ly.qkv[1]) &&
             qw(p + "self_attn.v_proj.weight", kv_dim, d->hidden, &ly.qkv[2]) &&
             qw(p + "self_attn.o_proj.weight", d->hidden, q_dim, &ly.o) &&
             qw(p + "mlp.gate_proj.weight", d->inter, d->hidden, &ly.gate) &&
             qw(p + "mlp.up_proj.weight", d->inter, d->hidden, &ly.up) &&
             qw(p + "mlp.down_proj.weight", d->hidden, d->inter, &ly.down) &&
             f32(p + "input_layernorm.weight", d->hidden, &ly.attn_norm, true) &&
             f32(p + "post_attention_layernorm.weight", d->hidden, &ly.ffn_norm, true) &&
             f32(p + "self_attn.q_proj.bias", q_dim, &ly.bias[0], false) &&
             f32(p + "self_attn.k_proj.bias", kv_dim, &ly.bias[1], false) &&
             f32(p + "self_attn.v_proj.bias", kv_dim, &ly.bias[2], false);
    }
    if (!ok) {
        const std::string msg = t_last_error;
        qraf_cuda_decoder_close(d.release());
        t_last_error = msg;
        return QRAF_ERR_INVALID;
    }
    // the LM head: lm_head.weight (quantized or F32), else the embedding (tied,
    // transformer.cpp:374-400)
    if (m->weights.count("lm_head.weight")) {
        if (!qw("lm_head.weight", d->vocab, d->hidden, &d->lm_head)) return fail_close(QRAF_ERR_INVALID, t_last_error);
    } else {
        const float* head = nullptr;
        f32("lm_head.weight", static_cast<uint64_t>(d->vocab) * d->hidden, &head, false);
        d->tied = true;
        d->lm_head.data = head ? head : d->emb;
    }
    DeviceInfo* dev = nullptr;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(d->device);
    rc = ensure_device(nullptr, &dev);
    if (rc) {
        cudaSetDevice(cur);
        const std::string msg = t_last_error;
        qraf_cuda_decoder_close(d.release());
        t_last_error = msg;
        return rc;
    }
    // attention: the largest partial buffer over steps of 1 .. max_slots slots
    uint64_t part_floats = 0;
    for (uint32_t M = 1; M <= max_slots; ++M) {
        const uint32_t S = attn_splits(d.get(), M, dev->sm_count);
        part_floats = std::max<uint64_t>(part_floats, static_cast<uint64_t>(M) * d->heads * S * (d->hd + 4u));
    }
    d->kv8 = (flags & QRAF_DECODER_KV_INT8) != 0;
    if (d->kv8 && d->hd % 16u) return fail_close(QRAF_ERR_UNSUPPORTED, "the int8 KV cache needs head_dim % 16 == 0");
    const size_t smem_max = d->kv8 ? attn_smem_bytes8(d->G, d->hd) : attn_smem_floats(d->G, d->hd) * sizeof(float);
    if (smem_max + kSmemReserve > static_cast<size_t>(dev->smem_optin)) {
        cudaSetDevice(cur);
        return fail_close(QRAF_ERR_UNSUPPORTED, "head_dim " + std::to_string(d->hd) + " with " + std::to_string(d->G) +
                                                    " query heads per KV head needs " + std::to_string(smem_max) +
                                                    " bytes of shared memory per CTA");
    }
    const uint64_t cache = static_cast<uint64_t>(max_slots) * d->layers * max_seq * kv_dim;
    const size_t ws = static_cast<size_t>(max_slots) * (2u * d->hidden + 2u * q_dim + 2u * kv_dim + 2u * d->inter);
    const size_t rope_n = static_cast<size_t>(max_seq) * (d->hd / 2u);
    const uint64_t scales = static_cast<uint64_t>(max_slots) * d->layers * max_seq * d->kv_heads;
    bool alloc_ok = d->kv8 ? (cudaMalloc(&d->kq, cache) == cudaSuccess && cudaMalloc(&d->vq, cache) == cudaSuccess &&
                              cudaMalloc(&d->ksc, scales * sizeof(float)) == cudaSuccess &&
                              cudaMalloc(&d->vsc, scales * sizeof(float)) == cudaSuccess)
                           : (cudaMalloc(&d->kc, cache * sizeof(float)) == cudaSuccess &&
                              cudaMalloc(&d->vc, cache * sizeof(float)) == cudaSuccess);
    alloc_ok = alloc_ok && cudaMalloc(&d->rope, rope_n * sizeof(float2)) == cudaSuccess &&
                    cudaMalloc(&d->part, std::max<uint64_t>(part_floats, 1) * sizeof(float)) == cudaSuccess &&
                    cudaMalloc(&d->counter, static_cast<size_t>(max_slots) * d->kv_heads * sizeof(uint32_t)) ==
                        cudaSuccess &&
                    cudaMalloc(&d->work, ws * sizeof(float)) == cudaSuccess;
    cudaError_t e = cudaSuccess;
    if (alloc_ok) {
        if (d->kv8) {   // QuantizedKVCache::init zero-fills codes and scales (kv_cache_quant.h:31-50)
            e = cudaMemset(d->kq, 0, cache);
            if (e == cudaSuccess) e = cudaMemset(d->vq, 0, cache);
            if (e == cudaSuccess) e = cudaMemset(d->ksc, 0, scales * sizeof(float));
            if (e == cudaSuccess) e = cudaMemset(d->vsc, 0, scales * sizeof(float));
        } else {
            e = cudaMemset(d->kc, 0, cache * sizeof(float));
            if (e == cudaSuccess) e = cudaMemset(d->vc, 0, cache * sizeof(float));
        }
        if (e == cudaSuccess)
            e = cudaMemset(d->counter, 0, static_cast<size_t>(max_slots) * d->kv_heads * sizeof(uint32_t));
        const uint32_t per = (d->G * (d->hd / 4u) + kAttnThreads - 1u) / kAttnThreads;   // quads per thread
        if (d->kv8)
            d->attn_kernel = per <= 1u ? dec_attention_kernel<1, true> : per <= 2u ? dec_attention_kernel<2, true>
                                                                                   : dec_attention_kernel<4, true>;
        else
            d->attn_kernel = per <= 1u ? dec_attention_kernel<1, false> : per <= 2u ? dec_attention_kernel<2, false>
                                                                                    : dec_attention_kernel<4, false>;
        if (e == cudaSuccess) e = cudaFuncSetAttribute(d->attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                       static_cast<int>(smem_max));
        if (e == cudaSuccess) {
            (dec_rope_table_kernel<<<static_cast<unsigned>(std::min<size_t>((rope_n + 255) / 256, 4u * dev->sm_count)),
                                     256>>>(d->rope, max_seq, d->hd, d->theta), count_launch());
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    cudaSetDevice(cur);
    if (!alloc_ok) {
        cudaGetLastError();
        return fail_close(QRAF_ERR_NOMEM, "the KV caches and work buffers (" +
                                              std::to_string((d->kv8 ? 2 * cache + 8 * scales : 8 * cache) + ws * 4 +
                                                             part_floats * 4) +
                                              " bytes) could not be allocated");
    }
    if (e != cudaSuccess) return fail_close(QRAF_ERR_CUDA, std::string("decoder set-up: ") + cudaGetErrorString(e));
    float* w = d->work;
    d->x = w;   w += static_cast<size_t>(max_slots) * d->hidden;
    d->q = w;   w += static_cast<size_t>(max_slots) * q_dim;
    d->k = w;   w += static_cast<size_t>(max_slots) * kv_dim;
    d->v = w;   w += static_cast<size_t>(max_slots) * kv_dim;
    d->att = w; w += static_cast<size_t>(max_slots) * q_dim;
    d->h = w;   w += static_cast<size_t>(max_slots) * d->inter;
    d->u = w;   w += static_cast<size_t>(max_slots) * d->inter;
    d->xn = w;
    // the tensor-core route: every projection tile-eligible, Q/K/V and gate/up contiguous
    auto joined = [](const qraf_weight_t* ws, uint32_t n, qraf_weight_t* out) {
        qraf_weight_t v = ws[0];
        for (uint32_t i = 1; i < n; ++i) {
            const uint8_t* end = static_cast<const uint8_t*>(ws[i - 1].data) + ws[i - 1].rows * ws[i - 1].row_bytes;
            if (ws[i].data != end || ws[i].dtype != v.dtype || ws[i].cols != v.cols || ws[i].block_size != v.block_size)
                return false;
            v.rows += ws[i].rows;
        }
        v.bytes = static_cast<uint64_t>(v.rows) * v.row_bytes;
        *out = v;
        return true;
    };
    bool tc = d->tied || tc_eligible(d->lm_head);
    for (uint32_t l = 0; tc && l < d->layers; ++l) {
        DecLayer& ly = d->L[l];
        const qraf_weight_t gu[2] = {ly.gate, ly.up};
        tc = joined(ly.qkv, 3, &ly.qkv_all) && joined(gu, 2, &ly.gate_up) && tc_eligible(ly.qkv_all) &&
             tc_eligible(ly.o) && tc_eligible(ly.gate_up) && tc_eligible(ly.down);
    }
    d->tc_route = tc;
    *out = d.release();
    return QRAF_OK;
}

int qraf_cuda_decoder_info(qraf_decoder_t d, uint32_t* vocab, uint32_t* hidden, uint32_t* layers, uint32_t* max_slots,
                           uint32_t* max_seq) {
    if (!d) return fail(QRAF_ERR_INVALID, "decoder is NULL");
    if (vocab) *vocab = d->vocab;
    if (hidden) *hidden = d->hidden;
    if (layers) *layers = d->layers;
    if (max_slots) *max_slots = d->max_slots;
    if (max_seq) *max_seq = d->max_seq;
    return QRAF_OK;
}

}  // extern "C"

namespace {

// The step on the tensor-core route: per layer four launch pairs (prep +
// tile) and the attention launch.  QKV: RMSNorm formed by the prep kernel,
// Q/K/V one weight with three outputs and their biases; O: the residual added
// by the tile's store; gate/up: RMSNorm in the prep, one weight, outputs gate
// and up; down: silu(gate) * up formed by the prep, the residual in the store;
// the LM head: the final RMSNorm in the prep.  The arithmetic is that of the
// separate passes (tests/test_gpu_decoder.py compares with the reference).
int tc_step(qraf_decoder* d, uint32_t M, const DeviceInfo* dev, AttnParams ap, cudaLaunchConfig_t cfg,
            float* logits_dev, cudaStream_t st) {
    const uint32_t q_dim = d->heads * d->hd, kv_dim = d->kv_heads * d->hd;
    int rc = QRAF_OK;
    for (uint32_t l = 0; l < d->layers; ++l) {
        const DecLayer& ly = d->L[l];
        TcFusion qkv;
        qkv.in.norm_w = ly.attn_norm;
        qkv.in.eps = d->eps;
        qkv.nseg = 3;
        float* outs[3] = {d->q, d->k, d->v};
        const uint32_t row0[kMaxSeg + 1] = {0u, q_dim, q_dim + kv_dim, q_dim + 2u * kv_dim, q_dim + 2u * kv_dim};
        for (int i = 0; i < 3; ++i) {
            qkv.seg_y[i] = outs[i];
            qkv.seg_b[i] = ly.bias[i];
        }
        for (int i = 0; i <= kMaxSeg; ++i) qkv.seg_row0[i] = row0[i];
        rc = matmul_tc(ly.qkv_all, d->x, nullptr, M, true, st, *dev, nullptr, 0, &qkv);
        if (rc) return rc;
        ap.layer = l;
        QRAF_CUDA_TRY(counted(cudaLaunchKernelEx(&cfg, d->attn_kernel, ap)));
        TcFusion res;
        res.accumulate = true;
        rc = matmul_tc(ly.o, d->att, d->x, M, true, st, *dev, nullptr, 0, &res);
        if (rc) return rc;
        TcFusion gu;
        gu.in.norm_w = ly.ffn_norm;
        gu.in.eps = d->eps;
        gu.nseg = 2;
        gu.seg_y[0] = d->h;
        gu.seg_y[1] = d->u;
        gu.seg_row0[1] = d->inter;
        for (int i = 2; i <= kMaxSeg; ++i) gu.seg_row0[i] = 2u * d->inter;
        rc = matmul_tc(ly.gate_up, d->x, nullptr, M, true, st, *dev, nullptr, 0, &gu);
        if (rc) return rc;
        TcFusion down;
        down.in.up = d->u;
        down.accumulate = true;
        rc = matmul_tc(ly.down, d->h, d->x, M, true, st, *dev, nullptr, 0, &down);
        if (rc) return rc;
    }
    if (!d->tied) {
        TcFusion head;
        head.in.norm_w = d->out_norm;
        head.in.eps = d->eps;
        return matmul_tc(d->lm_head, d->x, logits_dev, M, true, st, *dev, nullptr, 0, &head);
    }
    (rmsnorm_kernel<<<M, 256, 0, st>>>(d->x, d->out_norm, d->eps, d->hidden, d->xn, 0), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    const size_t warps = static_cast<size_t>(d->vocab) * M;
    (dec_f32_matvec_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
         static_cast<const float*>(d->lm_head.data), d->xn, d->vocab, d->hidden, M, logits_dev),
     count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

}  // namespace

extern "C" {

int qraf_cuda_decoder_kv_read(qraf_decoder_t d, uint32_t slot, uint32_t layer, uint32_t pos, void* k_out, void* v_out,
                              float* k_scales, float* v_scales) {
    if (!d) return fail(QRAF_ERR_INVALID, "decoder is NULL");
    if (slot >= d->max_slots || layer >= d->layers || pos >= d->max_seq)
        return fail(QRAF_ERR_INVALID, "slot %u, layer %u or position %u out of range", slot, layer, pos);
    if (!k_out || !v_out || (d->kv8 && (!k_scales || !v_scales)))
        return fail(QRAF_ERR_INVALID, "an output pointer is NULL");
    const uint32_t kv_dim = d->kv_heads * d->hd;
    const size_t row = ((static_cast<size_t>(slot) * d->layers + layer) * d->max_seq + pos) * kv_dim;
    const size_t srow = ((static_cast<size_t>(slot) * d->layers + layer) * d->max_seq + pos) * d->kv_heads;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(d->device);
    cudaError_t e;
    if (d->kv8) {
        e = cudaMemcpy(k_out, d->kq + row, kv_dim, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(v_out, d->vq + row, kv_dim, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(k_scales, d->ksc + srow, d->kv_heads * sizeof(float), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(v_scales, d->vsc + srow, d->kv_heads * sizeof(float), cudaMemcpyDeviceToHost);
    } else {
        e = cudaMemcpy(k_out, d->kc + row, kv_dim * sizeof(float), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(v_out, d->vc + row, kv_dim * sizeof(float), cudaMemcpyDeviceToHost);
    }
    cudaSetDevice(cur);
    if (e != cudaSuccess) return fail(QRAF_ERR_CUDA, "reading the KV cache: %s", cudaGetErrorString(e));
    return QRAF_OK;
}

int qraf_cuda_decoder_step(qraf_decoder_t d, uint32_t M, const int32_t* tokens_dev, const int32_t* pos_dev,
                           const int32_t* slots_dev, float* logits_dev, int mode, void* stream) {
    if (!d) return fail(QRAF_ERR_INVALID, "decoder is NULL");
    if (M == 0) return QRAF_OK;
    if (M > d->max_slots) return fail(QRAF_ERR_INVALID, "M = %u exceeds max_slots = %u", M, d->max_slots);
    if (!tokens_dev || !pos_dev || !slots_dev || !logits_dev) return fail(QRAF_ERR_INVALID, "a pointer is NULL");
    const int base_mode = mode & 0xFF;
    if (base_mode != QRAF_MODE_EXACT && base_mode != QRAF_MODE_FAST && base_mode != QRAF_MODE_TC &&
        base_mode != QRAF_MODE_AUTO)
        return fail(QRAF_ERR_INVALID, "unknown mode %d", mode);
    const int pmode = base_mode | QRAF_MODE_FLAG_OVERLAP;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    DeviceInfo* dev = nullptr;
    int cur = 0;
    int rc = ensure_device(&cur, &dev);
    if (rc) return rc;
    if (cur != d->device)
        return fail(QRAF_ERR_INVALID, "the decoder lives on device %d, the current device is %d", d->device, cur);
    const uint32_t S = attn_splits(d, M, dev->sm_count);
    AttnParams ap{};
    ap.q = d->q;
    ap.k = d->k;
    ap.v = d->v;
    ap.rope = d->rope;
    ap.pos = pos_dev;
    ap.slots = slots_dev;
    ap.kc = d->kc;
    ap.vc = d->vc;
    ap.kq = d->kq;
    ap.vq = d->vq;
    ap.ksc = d->ksc;
    ap.vsc = d->vsc;
    ap.out = d->att;
    ap.part = d->part;
    ap.counter = d->counter;
    ap.heads = d->heads;
    ap.kv_heads = d->kv_heads;
    ap.hd = d->hd;
    ap.G = d->G;
    ap.layers = d->layers;
    ap.max_seq = d->max_seq;
    ap.max_slots = d->max_slots;
    ap.scale = 1.0f / std::sqrt(static_cast<float>(d->hd));   // attention.cpp:118, IEEE on the host as there
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, d->kv_heads, M);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = d->kv8 ? attn_smem_bytes8(d->G, d->hd) : attn_smem_floats(d->G, d->hd) * sizeof(float);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;

    (dec_embed_kernel<<<M, 256, 0, st>>>(d->emb, tokens_dev, d->vocab, d->hidden, d->x), count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    const bool tc = d->tc_route && M >= 2 &&
                    (base_mode == QRAF_MODE_TC || (base_mode == QRAF_MODE_AUTO && M >= kAutoTcMinVectors));
    if (tc) return tc_step(d, M, dev, ap, cfg, logits_dev, st);
    for (uint32_t l = 0; l < d->layers; ++l) {
        const DecLayer& ly = d->L[l];
        float* qkv_out[3] = {d->q, d->k, d->v};
        const float* biases[3] = {ly.bias[0], ly.bias[1], ly.bias[2]};
        const bool any_bias = biases[0] || biases[1] || biases[2];
        rc = multi_impl(ly.qkv, 3, d->x, ly.attn_norm, d->eps, any_bias ? biases : nullptr, qkv_out, M, pmode, st);
        if (rc) return rc;
        ap.layer = l;
        QRAF_CUDA_TRY(counted(cudaLaunchKernelEx(&cfg, d->attn_kernel, ap)));
        rc = matvec_impl(&ly.o, d->att, d->x, M, pmode, st, true);
        if (rc) return rc;
        rc = swiglu_impl(&ly.gate, &ly.up, d->x, ly.ffn_norm, d->eps, d->h, M, pmode, st);
        if (rc) return rc;
        rc = matvec_impl(&ly.down, d->h, d->x, M, pmode, st, true);
        if (rc) return rc;
    }
    if (!d->tied) {
        float* outs[1] = {logits_dev};
        return multi_impl(&d->lm_head, 1, d->x, d->out_norm, d->eps, nullptr, outs, M, pmode, st);
    }
    (rmsnorm_kernel<<<M, 256, 0, st>>>(d->x, d->out_norm, d->eps, d->hidden, d->xn, base_mode == QRAF_MODE_EXACT),
     count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    const size_t warps = static_cast<size_t>(d->vocab) * M;
    (dec_f32_matvec_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, st>>>(
         static_cast<const float*>(d->lm_head.data), d->xn, d->vocab, d->hidden, M, logits_dev),
     count_launch());
    QRAF_CUDA_TRY(cudaGetLastError());
    return QRAF_OK;
}

}  // extern "C"
