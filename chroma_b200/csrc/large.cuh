// Kernels of the large-width bf16 path (GPT-OSS-20B/120B shapes): everything around the tensor-core GEMMs
// (gemm.cuh) and flash attention (flash.cuh). Activations are bf16 like the exported graph's values; each kernel
// rounds where the reference rounds (chroma/_src/lowering.py:185-210, gpt_oss.py).
//
//   k_embed_bf16    embedding rows -> residual stream x                       (gpt_oss.py:304-306)
//   k_rms_bf16      x -> bf16(x * rsqrt(mean(x^2) + eps) * w)                 (gpt_oss.py:30-41)
//   k_rope_split    fused QKV output -> q (RoPE), new K rows (RoPE), new V rows (gpt_oss.py:44-54, 189-202)
//   k_router        gate logits -> top-k experts (sorted, lowest index on ties) + softmax weights (gpt_oss.py:246-247)
//   k_route_count / k_route_offsets / k_route_scatter
//                   group the (token, slot) pairs by expert: counts, row offsets, and the gathered expert inputs
//   k_moe_combine   x += bf16(sum_s w[t,s] * y[row(t,s)])                     (gpt_oss.py:263-265)
//   k_norm_rows     final RMSNorm of the rows whose logits are wanted (fp32 and bf16 copies)
//   k_argmax_rows   greedy argmax keys over bf16 logits rows
#pragma once

#include "gptoss.cuh"

namespace cb200 {

using bf16 = __nv_bfloat16;

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

// grid = tokens; block = 256. qkv [N][(H+2KV)*hd] -> q [N][H][hd] (RoPE), k_out/v_out rows [N][KV][hd].
__global__ void __launch_bounds__(256) k_rope_split(const bf16* __restrict__ qkv, int H, int KV, int hd,
                                                    const float* __restrict__ positions, const float* __restrict__ inv_freq,
                                                    float conc, bf16* __restrict__ q, bf16* __restrict__ k_out,
                                                    bf16* __restrict__ v_out) {
    const int t = blockIdx.x;
    const int half = hd / 2, heads = H + 2 * KV;
    pdl_wait();
    pdl_trigger();
    const float pos = positions[t];
    const bf16* row = qkv + size_t(t) * heads * hd;
    for (int i = threadIdx.x; i < heads * half; i += blockDim.x) {
        const int hh = i / half, j = i % half;
        const float lo = __bfloat162float(row[hh * hd + j]), hi = __bfloat162float(row[hh * hd + j + half]);
        float o1 = lo, o2 = hi;
        if (hh < H + KV) {
            float s, c;
            sincosf(__fmul_rn(pos, inv_freq[j]), &s, &c);
            c = bf16_round(__fmul_rn(c, conc));
            s = bf16_round(__fmul_rn(s, conc));
            o1 = bf16_round(__fsub_rn(bf16_round(__fmul_rn(lo, c)), bf16_round(__fmul_rn(hi, s))));
            o2 = bf16_round(__fadd_rn(bf16_round(__fmul_rn(hi, c)), bf16_round(__fmul_rn(lo, s))));
        }
        bf16* dst = hh < H ? q + (size_t(t) * H + hh) * hd
                           : (hh < H + KV ? k_out + (size_t(t) * KV + hh - H) * hd : v_out + (size_t(t) * KV + hh - H - KV) * hd);
        dst[j] = __float2bfloat16_rn(o1);
        dst[j + half] = __float2bfloat16_rn(o2);
    }
}

// One warp per token: gate logits [N][E] (bf16) -> sorted top-k indices and softmax weights.
__global__ void k_router(const bf16* __restrict__ logits, int ntok, int E, int k, int* __restrict__ ridx,
                         float* __restrict__ rw, int* __restrict__ routes) {
    __shared__ float g[8][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    pdl_wait();
    pdl_trigger();
    if (t >= ntok) return;
    for (int e = lane; e < E; e += 32) g[warp][e] = __bfloat162float(logits[size_t(t) * E + e]);
    __syncwarp();
    warp_topk_softmax<bf16>(g[warp], E, k, ridx + size_t(t) * k, rw + size_t(t) * k);
    __syncwarp();
    if (routes && lane < k) routes[size_t(t) * k + lane] = ridx[size_t(t) * k + lane];
}

__global__ void k_route_count(const int* __restrict__ ridx, int pairs, int* __restrict__ counts) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < pairs) atomicAdd(counts + ridx[i], 1);
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
    for (int c = lane; c < d / 8; c += 32) dst[c] = src[c];
}

// grid = tokens; x[t] = bf16(x[t] + bf16(sum_s w[t,s] * y[perm[t,s]])) summed in slot order (perm == nullptr:
// y row t*k + s, the layout of the expert-parallel return buffer).
__global__ void __launch_bounds__(256) k_moe_combine(const bf16* __restrict__ y, const int* __restrict__ perm,
                                                     const float* __restrict__ rw, int k, int d, bf16* __restrict__ x) {
    const int t = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    int rows[8];
    float w[8];
    for (int s = 0; s < k; ++s) {
        rows[s] = perm ? perm[size_t(t) * k + s] : t * k + s;
        w[s] = rw[size_t(t) * k + s];
    }
    for (int c = threadIdx.x * 2; c < d; c += blockDim.x * 2) {
        float a0 = 0.f, a1 = 0.f;
        for (int s = 0; s < k; ++s) {
            const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(y + size_t(rows[s]) * d + c));
            a0 = __fadd_rn(a0, __fmul_rn(v.x, w[s]));
            a1 = __fadd_rn(a1, __fmul_rn(v.y, w[s]));
        }
        __nv_bfloat162* xp = reinterpret_cast<__nv_bfloat162*>(x + size_t(t) * d + c);
        const float2 xv = __bfloat1622float2(*xp);
        *xp = __floats2bfloat162_rn(bf16_round(xv.x + bf16_round(a0)), bf16_round(xv.y + bf16_round(a1)));
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

// One CTA per row of bf16 logits: argmax key (larger value, then lower index).
__global__ void __launch_bounds__(1024) k_argmax_rows(const bf16* __restrict__ logits, int V, unsigned long long* __restrict__ keys) {
    __shared__ unsigned long long red[32];
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    unsigned long long best = 0ull;
    const bf16* row = logits + size_t(r) * V;
    for (int v = threadIdx.x; v < V; v += blockDim.x) best = max(best, argmax_key(__bfloat162float(row[v]), v));
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (lane == 0) red[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < warps; ++w) best = max(best, red[w]);
        keys[r] = max(best, red[0]);
    }
}

}  // namespace cb200
