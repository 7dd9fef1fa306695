// Kernels of the large-width bf16 path (GPT-OSS-20B/120B shapes): everything around the tensor-core GEMMs
// (gemm.cuh) and flash attention (flash.cuh). Activations are bf16 like the exported graph's values; each kernel
// rounds where the reference rounds (chroma/_src/lowering.py:185-210, gpt_oss.py).
//
//   k_embed_bf16    embedding rows -> residual stream x                       (gpt_oss.py:304-306)
//   k_rms_bf16      x -> bf16(x * rsqrt(mean(x^2) + eps) * w)                 (gpt_oss.py:30-41)
//   k_rope_split    fused QKV output -> q (RoPE), new K rows (RoPE), new V rows (gpt_oss.py:44-54, 189-202); where
//                   the QKV GEMM has no split-K, its kEpiRope epilogue does this instead from k_rope_table's pairs
//   k_route_fused   norm -> gate logits -> top-k experts (sorted, lowest index on ties) + softmax weights, and the
//                   per-expert counts (gpt_oss.py:243-247)
//   k_route_offsets / k_route_scatter
//                   group the (token, slot) pairs by expert: row offsets and the gathered expert inputs
//   k_moe_combine   x += bf16(sum_s w[t,s] * y[row(t,s)]) (gpt_oss.py:263-265), optionally the next layer's norm
//   k_norm_rows     final RMSNorm of the rows whose logits are wanted (fp32 and bf16 copies)
#pragma once

#include "gptoss.cuh"

namespace cb200 {

using bf16 = __nv_bfloat16;
constexpr int kEpMaxGate = 256;  // most experts a router ranks

__global__ void k_embed_bf16(const int64_t* __restrict__ tokens, int ntok, const bf16* __restrict__ emb, int V, int d,
                             bf16* __restrict__ x, unsigned* err) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= ntok) return;
    const int64_t row = checked_row(tokens[t], V, false, err);
    const uint4* src = reinterpret_cast<const uint4*>(emb + size_t(row) * d);
    uint4* dst = reinterpret_cast<uint4*>(x + size_t(t) * d);
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) dst[c] = src[c];
}

// One CTA per row; d a multiple of 8.
__global__ void __launch_bounds__(256) k_rms_bf16(const bf16* __restrict__ x, int d, float eps, const float* __restrict__ w,
                                                  bf16* __restrict__ out) {
    __shared__ float red[32];
    const size_t r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    const bf16* xr = x + r * d;
    float s = 0.f;
    for (int c = threadIdx.x * 2; c < d; c += blockDim.x * 2) {
        const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + c));
        s = fmaf(v.x, v.x, s);
        s = fmaf(v.y, v.y, s);
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float t = lane < warps ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = 1.0f / sqrtf(t / float(d) + eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int c = threadIdx.x * 2; c < d; c += blockDim.x * 2) {
        const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + c));
        *reinterpret_cast<__nv_bfloat162*>(out + r * d + c) =
            __floats2bfloat162_rn(__fmul_rn(__fmul_rn(v.x, inv), w[c]), __fmul_rn(__fmul_rn(v.y, inv), w[c + 1]));
    }
}

// grid = tokens; block = 256. qkv [N][(H+2KV)*hd] -> q [N][H][hd] (RoPE), k_out/v_out rows [N][KV][hd]. The hd/2
// (cos, sin) pairs of the token's position are computed once into shared memory (rounded like the reference's
// cos/sin tensors, gpt_oss.py:44-54); each thread then rotates two adjacent (lo, hi) pairs with 4-byte accesses.
__global__ void __launch_bounds__(256) k_rope_split(const bf16* __restrict__ qkv, int H, int KV, int hd,
                                                    const float* __restrict__ positions, const float* __restrict__ inv_freq,
                                                    float conc, bf16* __restrict__ q, bf16* __restrict__ k_out,
                                                    bf16* __restrict__ v_out) {
    __shared__ float cs[64][2];
    const int t = blockIdx.x;
    const int half = hd / 2, heads = H + 2 * KV;
    pdl_wait();
    pdl_trigger();
    const float pos = positions[t];
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
        float sn, c;
        sincosf(__fmul_rn(pos, inv_freq[j]), &sn, &c);
        cs[j][0] = bf16_round(__fmul_rn(c, conc));
        cs[j][1] = bf16_round(__fmul_rn(sn, conc));
    }
    __syncthreads();
    const bf16* row = qkv + size_t(t) * heads * hd;
    const int pairs2 = half / 2;  // 2 rotation pairs per thread step
    for (int i = threadIdx.x; i < heads * pairs2; i += blockDim.x) {
        const int hh = i / pairs2, j = (i % pairs2) * 2;
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(row + hh * hd + j));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(row + hh * hd + j + half));
        float o1[2] = {lo.x, lo.y}, o2[2] = {hi.x, hi.y};
        if (hh < H + KV) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float c = cs[j + u][0], sn = cs[j + u][1];
                const float l = u ? lo.y : lo.x, h = u ? hi.y : hi.x;
                o1[u] = bf16_round(__fsub_rn(bf16_round(__fmul_rn(l, c)), bf16_round(__fmul_rn(h, sn))));
                o2[u] = bf16_round(__fadd_rn(bf16_round(__fmul_rn(h, c)), bf16_round(__fmul_rn(l, sn))));
            }
        }
        bf16* dst = hh < H ? q + (size_t(t) * H + hh) * hd
                           : (hh < H + KV ? k_out + (size_t(t) * KV + hh - H) * hd : v_out + (size_t(t) * KV + hh - H - KV) * hd);
        *reinterpret_cast<__nv_bfloat162*>(dst + j) = __floats2bfloat162_rn(o1[0], o1[1]);
        *reinterpret_cast<__nv_bfloat162*>(dst + j + half) = __floats2bfloat162_rn(o2[0], o2[1]);
    }
}

// (cos, sin) of every token's position for the QKV GEMM's RoPE epilogue (kEpiRope), once per forward: cs[t * half + j]
// = the pair k_rope_split computes for token t and frequency j, rounded the same way.
__global__ void k_rope_table(const float* __restrict__ positions, const float* __restrict__ inv_freq, float conc,
                             int ntok, int half, float2* __restrict__ cs) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= ntok * half) return;
    float sn, c;
    sincosf(__fmul_rn(positions[i / half], inv_freq[i % half]), &sn, &c);
    cs[i] = make_float2(bf16_round(__fmul_rn(c, conc)), bf16_round(__fmul_rn(sn, conc)));
}

// One warp per token: gate logits [N][E] (bf16, from the tensor-core gate GEMM) -> sorted top-k experts, softmax
// weights, per-expert counts and the optional routing record (the many-token counterpart of k_route_fused).
__global__ void __launch_bounds__(256) k_route_topk(const bf16* __restrict__ logits, int ntok, int E, int k,
                                                    int* __restrict__ ridx, float* __restrict__ rw,
                                                    int* __restrict__ routes, int* __restrict__ counts) {
    __shared__ float g[8][kEpMaxGate];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    pdl_wait();
    pdl_trigger();
    if (t >= ntok) return;
    for (int e = lane; e < E; e += 32) g[warp][e] = __bfloat162float(logits[size_t(t) * E + e]);
    __syncwarp();
    int* ri = ridx + size_t(t) * k;
    warp_topk_softmax<bf16>(g[warp], E, k, ri, rw + size_t(t) * k);
    __syncwarp();
    if (lane < k) {
        const int e = ri[lane];
        atomicAdd(counts + e, 1);
        if (routes) routes[size_t(t) * k + lane] = e;
    }
}

// Single CTA: offsets[e] = exclusive prefix sum of counts; cursor[e] = offsets[e]; counts cleared for the next layer.
__global__ void k_route_offsets(int* __restrict__ counts, int E, int* __restrict__ offsets, int* __restrict__ cursor) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            offsets[e] = acc;
            cursor[e] = acc;
            acc += counts[e];
            counts[e] = 0;
        }
        offsets[E] = acc;
    }
}

// One warp per (token, slot): claim a row in its expert's group and copy the token's normalised activations there.
__global__ void k_route_scatter(const int* __restrict__ ridx, int pairs, int k, int d, const bf16* __restrict__ xn,
                                int* __restrict__ cursor, int* __restrict__ perm, bf16* __restrict__ grouped) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.x * (blockDim.x >> 5) + warp;
    pdl_wait();
    pdl_trigger();
    if (i >= pairs) return;
    int row = 0;
    if (lane == 0) {
        row = atomicAdd(cursor + ridx[i], 1);
        perm[i] = row;
    }
    row = __shfl_sync(0xffffffffu, row, 0);
    const uint4* src = reinterpret_cast<const uint4*>(xn + size_t(i / k) * d);
    uint4* dst = reinterpret_cast<uint4*>(grouped + size_t(row) * d);
#pragma unroll 4
    for (int c = lane; c < d / 8; c += 32) dst[c] = src[c];
}

// Optional duties of k_moe_combine: wait for the expert outputs other GPUs return (expert parallel), and the next
// layer's attention RMSNorm of the updated row (saves a launch and a re-read of x).
struct CombineExtra {
    const unsigned* wait_flags;  // [wait_count] flags, each must reach *wait_epoch; nullptr: no wait
    int wait_count;
    const unsigned* wait_epoch;
    unsigned long long wait_timeout_ns;
    unsigned* err;
    const float* norm_w;  // next layer's attention norm scale, or nullptr
    float eps;
    bf16* xn;             // [tokens][d] normalised rows
};

// grid = tokens; x[t] = bf16(x[t] + bf16(sum_s w[t,s] * y[perm[t,s]])) summed in slot order (perm == nullptr:
// y row t*k + s, the layout of the expert-parallel return buffer). With ex.norm_w, also xn[t] = bf16(x[t] * inv * w)
// with inv = 1/sqrt(mean(x[t]^2) + eps) (the sum of squares in another order than k_rms_bf16's).
__global__ void __launch_bounds__(256) k_moe_combine(const bf16* __restrict__ y, const int* __restrict__ perm,
                                                     const float* __restrict__ rw, int k, int d, bf16* __restrict__ x,
                                                     CombineExtra ex) {
    __shared__ float red[32];
    __shared__ int ok;
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    if (ex.wait_flags) {
        if (threadIdx.x == 0) ok = 1;
        __syncthreads();
        if (int(threadIdx.x) < ex.wait_count &&
            !wait_flag_geq(ex.wait_flags + threadIdx.x, *reinterpret_cast<const volatile unsigned*>(ex.wait_epoch),
                           ex.wait_timeout_ns, ex.err))
            ok = 0;
        __syncthreads();
        if (!ok) return;
    }
    int rows[8];
    float w[8];
    for (int s = 0; s < k; ++s) {
        rows[s] = perm ? perm[size_t(t) * k + s] : t * k + s;
        w[s] = rw[size_t(t) * k + s];
    }
    // 8 columns per thread per step (16-byte loads of the k expert rows and of x); d is a multiple of 8.
    float sq = 0.f;
    for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < k; ++s) {
            const uint4 u = *reinterpret_cast<const uint4*>(y + size_t(rows[s]) * d + c);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 v = __bfloat1622float2(h[j]);
                a[2 * j] = __fadd_rn(a[2 * j], __fmul_rn(v.x, w[s]));
                a[2 * j + 1] = __fadd_rn(a[2 * j + 1], __fmul_rn(v.y, w[s]));
            }
        }
        uint4* xp = reinterpret_cast<uint4*>(x + size_t(t) * d + c);
        uint4 xu = *xp;
        __nv_bfloat162* xh = reinterpret_cast<__nv_bfloat162*>(&xu);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 xv = __bfloat1622float2(xh[j]);
            const float n0 = bf16_round(xv.x + bf16_round(a[2 * j])), n1 = bf16_round(xv.y + bf16_round(a[2 * j + 1]));
            xh[j] = __floats2bfloat162_rn(n0, n1);
            sq = fmaf(n0, n0, sq);
            sq = fmaf(n1, n1, sq);
        }
        *xp = xu;
    }
    if (!ex.norm_w) return;
    sq = warp_sum(sq);
    if (lane == 0) red[warp] = sq;
    __syncthreads();
    if (warp == 0) {
        float tot = lane < warps ? red[lane] : 0.f;
        tot = warp_sum(tot);
        if (lane == 0) red[0] = 1.0f / sqrtf(tot / float(d) + ex.eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {  // each thread re-reads the columns it wrote
        uint4 u = *reinterpret_cast<const uint4*>(x + size_t(t) * d + c);
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 v = __bfloat1622float2(h[j]);
            h[j] = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(v.x, inv), ex.norm_w[c + 2 * j]),
                                         __fmul_rn(__fmul_rn(v.y, inv), ex.norm_w[c + 2 * j + 1]));
        }
        *reinterpret_cast<uint4*>(ex.xn + size_t(t) * d + c) = u;
    }
}

// Final RMSNorm of selected rows (rows[s] = row within sequence s, negative wraps; nullptr = every row) into an
// fp32 copy (SIMT vocab kernel) and a bf16 copy (tensor-core vocab GEMM); clears the argmax keys.
__global__ void __launch_bounds__(256) k_norm_rows(const bf16* __restrict__ x, int nrows, const int64_t* __restrict__ rows,
                                                   int rows_per_seq, const float* __restrict__ w, int d, float eps,
                                                   float* __restrict__ out32, bf16* __restrict__ out16,
                                                   unsigned long long* __restrict__ keys, unsigned* err) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    int64_t src = r;
    if (rows != nullptr) src = int64_t(r) * rows_per_seq + checked_row(rows[r], rows_per_seq, true, err);
    const bf16* xr = x + size_t(src) * d;
    float s = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float v = __bfloat162float(xr[c]);
        s = fmaf(v, v, s);
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int i = 0; i < warps; ++i) tot += red[i];
        red[0] = 1.0f / sqrtf(tot / float(d) + eps);
        if (keys) keys[r] = 0ull;
    }
    __syncthreads();
    const float inv = red[0];
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float v = bf16_round(__fmul_rn(__fmul_rn(__bfloat162float(xr[c]), inv), w[c]));
        out32[size_t(r) * d + c] = v;
        out16[size_t(r) * d + c] = __float2bfloat16_rn(v);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// MoE routing in one launch: RMSNorm of the residual rows (-> xn, the experts' input), gate logits (bf16, + bias),
// top-k with softmax weights, and the per-expert counts the grouping needs (gpt_oss.py:243-247).
// grid = (ceil(ntok / 8), ceil(E / epc)); block = kThreads. CTA (tile, eb) normalises its 8 rows and computes gate
// logits for experts [epc eb, epc eb + epc) (one weight row per warp at a time, register-resident fragments); the
// last CTA of the token tile to finish (atomic counter, reset by it) runs top-k over all E logits of its rows. Many
// token tiles: epc = E (no redundant norms); few (decode): small epc spreads the gate weights over more SMs.

__global__ void __launch_bounds__(kThreads) k_route_fused(const bf16* __restrict__ x, int ntok, int d, float eps,
                                                          const float* __restrict__ norm_w, const bf16* __restrict__ gate_w,
                                                          const bf16* __restrict__ gate_b, int E, int epc, int k,
                                                          bf16* __restrict__ xn, bf16* __restrict__ glog,
                                                          int* __restrict__ ridx, float* __restrict__ rw,
                                                          int* __restrict__ routes, int* __restrict__ counts,
                                                          unsigned* __restrict__ tile_counters) {
    extern __shared__ float rsm[];
    constexpr int TT = kTileTokens, MR = 1;
    float* xs = rsm;               // [TT][d]
    float* gl = xs + TT * d;       // [TT][E]
    float* inv = gl + TT * E;      // [TT]
    __shared__ bool s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * TT, tt = min(TT, ntok - t0);
    const int e_begin = blockIdx.y * epc, e_end = min(E, e_begin + epc);
    // This warp's first two expert rows: loaded before waiting on the producer of x (weights only).
    int e0 = e_begin + warp * MR;
    const bf16* rows[MR] = {gate_w + size_t(min(e0, E - 1)) * d};
    Frag<MR> f;
    frag_load<bf16, MR>(f, rows, max(0, min(MR, e_end - e0)), d, 0);
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x * 8; i < tt * d; i += blockDim.x * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(x + size_t(t0) * d + i);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f2 = __bfloat1622float2(h[j]);
            xs[i + 2 * j] = f2.x;
            xs[i + 2 * j + 1] = f2.y;
        }
    }
    __syncthreads();
    // RMSNorm: same arithmetic as k_rms_bf16 (fp32 sum of squares, bf16(x * inv * w)).
    rows_rmsnorm<bf16>(xs, tt, d, eps, norm_w, inv);
    if (blockIdx.y == 0)
        for (int i = threadIdx.x * 2; i < tt * d; i += blockDim.x * 2)
            *reinterpret_cast<__nv_bfloat162*>(xn + size_t(t0) * d + i) = __floats2bfloat162_rn(xs[i], xs[i + 1]);
    for (; e0 < e_end; e0 += kWarps * MR) {
        const int nr = min(MR, e_end - e0);
        if (e0 != e_begin + warp * MR) {
            rows[0] = gate_w + size_t(e0) * d;
            frag_load<bf16, MR>(f, rows, nr, d, 0);
        }
        float acc[MR][TT];
        warp_gemv<bf16, MR, TT>(f, rows, nr, xs, d, tt, acc);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                if (r >= nr) break;
                const float b = __bfloat162float(gate_b[e0 + r]);
#pragma unroll
                for (int t = 0; t < TT; ++t)
                    if (t < tt) glog[size_t(t0 + t) * E + e0 + r] = __float2bfloat16_rn(__fadd_rn(acc[r][t], b));
            }
        }
    }
    // Last expert block of this token tile: top-k over all E gate logits of each row.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        bool last = true;
        if (gridDim.y > 1) {
            const unsigned prev = atomicAdd(tile_counters + blockIdx.x, 1u);
            last = prev == gridDim.y - 1;
            if (last) tile_counters[blockIdx.x] = 0u;
        }
        s_last = last;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < tt * E; i += blockDim.x) gl[i] = __bfloat162float(__ldcg(glog + size_t(t0) * E + i));
    __syncthreads();
    for (int t = warp; t < tt; t += kWarps) {
        int* ri = ridx + size_t(t0 + t) * k;
        warp_topk_softmax<bf16>(gl + t * E, E, k, ri, rw + size_t(t0 + t) * k);
        __syncwarp();
        if (lane < k) {
            const int e = ri[lane];
            atomicAdd(counts + e, 1);
            if (routes) routes[size_t(t0 + t) * k + lane] = e;
        }
    }
}

}  // namespace cb200
