// GPT-OSS-style transformer kernels (fp32 or bf16 storage) for token counts up to a few hundred per launch.
//
// One fused kernel per stage of the block, replacing the reference's chain of generated one-thread-per-element
// kernels plus cuBLAS calls (chroma/_src/codegen/gpu.py:165-424, chroma/_src/codegen/cuda/codegen.py:87-140):
//
//   k_embed         embedding gather with bounds check                         (gpt_oss.py:304-306)
//   k_attn_in       RMSNorm -> QKV linear (+bias) -> RoPE -> q, new K/V rows   (gpt_oss.py:189-202)
//   k_attention     scores*scale + mask, sink column, softmax, P.V            (gpt_oss.py:133-151, cached.py:36-47)
//   k_out_router    out linear + residual -> RMSNorm -> gate -> top-k -> softmax (gpt_oss.py:204-209, 243-247)
//   k_moe_up        selected-expert mlp1 GEMV (+bias) -> interleaved SwiGLU   (gpt_oss.py:251-254, 212-219)
//   k_moe_down      selected-expert mlp2 GEMV (+bias) -> weighted combine -> residual (gpt_oss.py:257-265)
//   k_final_norm    final RMSNorm of the rows whose logits are wanted         (gpt_oss.py:309, cached.py:50)
//   k_vocab         unembedding GEMV, the 201,088-way vocab projection        (gpt_oss.py:310)
//
// Activations live in fp32 buffers; for bf16 programs every value is rounded to bf16 wherever the exported graph
// rounds it (after each linear, einsum, residual add and SwiGLU step), so results track the reference's CPU program.
#pragma once

#include "common.cuh"

namespace cb200 {

struct Dims {
    int d, H, KV, hd, G, E, k, I, V;
    float eps, sm_scale, alpha, limit, conc;
};

template <typename T> struct LayerW {
    const float* attn_norm;
    const T* sinks;
    const T* qkv_w;
    const T* qkv_b;
    const T* out_w;
    const T* out_b;
    const float* mlp_norm;
    const T* gate_w;
    const T* gate_b;
    const T* w1;
    const T* b1;
    const T* w2;
    const T* b2;
};

enum MaskMode : int { kMaskBuffer = 0, kMaskCausal = 1, kMaskSlots = 2 };

// ------------------------------------------------------------------------------------------------------
// Block-wide RMS of rows held in shared memory: one warp per row. inv[r] = 1 / sqrt(sum(x^2)/d + eps),
// the fused norm of chroma/_src/codegen/cpu/kernels.h:101-115.
__device__ __forceinline__ void rows_inv_rms(const float* xs, int rows, int d, float eps, float* inv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int r = warp; r < rows; r += warps) {
        float s = 0.f;
        for (int c = lane; c < d; c += 32) s = fmaf(xs[r * d + c], xs[r * d + c], s);
        s = warp_sum(s);
        if (lane == 0) inv[r] = 1.0f / sqrtf(s / float(d) + eps);
    }
}

// Dot product of one weight row (length d, storage T, 16/8-byte aligned) with `tt` fp32 rows in shared
// memory (row stride d), accumulated by the whole warp; result valid in every lane.
template <typename T, int MAXT>
__device__ __forceinline__ void warp_row_dots(const T* wrow, const float* xs, int d, int tt, float (&acc)[MAXT]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < MAXT; ++t) acc[t] = 0.f;
    for (int c = lane * 4; c < d; c += 128) {
        float w4[4];
        load4(wrow + c, w4);
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            if (t < tt) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + t * d + c);
                acc[t] = fmaf(w4[0], xv.x, acc[t]);
                acc[t] = fmaf(w4[1], xv.y, acc[t]);
                acc[t] = fmaf(w4[2], xv.z, acc[t]);
                acc[t] = fmaf(w4[3], xv.w, acc[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < MAXT; ++t) acc[t] = warp_sum(acc[t]);
}

// ------------------------------------------------------------------------------------------------------
template <typename T>
__global__ void k_embed(const int64_t* tokens, int ntok, const T* emb, int V, int d, float* x, unsigned* err) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= ntok) return;
    const int64_t row = checked_row(tokens[t], V, false, err);
    const T* src = emb + size_t(row) * d;
    for (int c = threadIdx.x; c < d; c += blockDim.x) x[size_t(t) * d + c] = Store<T>::load(src + c);
}

// ------------------------------------------------------------------------------------------------------
// grid = (ceil(heads_total / hpc), ceil(ntok / TT)); block = 256. Each CTA owns `hpc` whole heads of the fused
// QKV projection (so RoPE pairs stay local) for up to TT tokens.
constexpr int kAttnInTokens = 8;

template <typename T>
__global__ void __launch_bounds__(256) k_attn_in(const float* __restrict__ x, int ntok, Dims dm, int hpc,
                                                 const float* __restrict__ norm_w, const T* __restrict__ W,
                                                 const T* __restrict__ bias, const float* __restrict__ positions,
                                                 const float* __restrict__ inv_freq, float* __restrict__ q_out,
                                                 T* __restrict__ k_out, T* __restrict__ v_out) {
    extern __shared__ float smem[];
    constexpr int TT = kAttnInTokens;
    const int d = dm.d, hd = dm.hd;
    const int heads_total = dm.H + 2 * dm.KV;
    const int head0 = blockIdx.x * hpc;
    const int nheads = min(hpc, heads_total - head0);
    const int cols = nheads * hd;
    const int t0 = blockIdx.y * TT;
    const int tt = min(TT, ntok - t0);
    float* xs = smem;                 // [TT][d]
    float* out = xs + TT * d;         // [TT][hpc*hd]
    float* inv = out + TT * hpc * hd; // [TT]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;

    prefetch_l2(W + size_t(head0) * hd * d, size_t(cols) * d * sizeof(T), threadIdx.x, blockDim.x);
    pdl_wait();
    pdl_trigger();

    for (int i = threadIdx.x; i < tt * d; i += blockDim.x) xs[i] = x[size_t(t0) * d + i];
    __syncthreads();
    rows_inv_rms(xs, tt, d, dm.eps, inv);
    __syncthreads();
    for (int i = threadIdx.x; i < tt * d; i += blockDim.x) {
        const int r = i / d, c = i % d;
        xs[i] = Store<T>::round(__fmul_rn(__fmul_rn(xs[i], inv[r]), norm_w[c]));
    }
    __syncthreads();

    for (int c = warp; c < cols; c += warps) {
        const int col = head0 * hd + c;
        float acc[TT];
        warp_row_dots<T, TT>(W + size_t(col) * d, xs, d, tt, acc);
        if (lane == 0) {
            const float b = Store<T>::load(bias + col);
#pragma unroll
            for (int t = 0; t < TT; ++t)
                if (t < tt) out[t * (hpc * hd) + c] = Store<T>::round(__fadd_rn(acc[t], b));
        }
    }
    __syncthreads();

    // RoPE on q and k heads (gpt_oss.py:44-54): o1 = x1*cos - x2*sin, o2 = x2*cos + x1*sin, cos/sin rounded to
    // storage first; v heads pass through.
    const int half = hd / 2;
    for (int i = threadIdx.x; i < tt * nheads * half; i += blockDim.x) {
        const int t = i / (nheads * half);
        const int rem = i % (nheads * half);
        const int lh = rem / half, j = rem % half;
        const int gh = head0 + lh;
        const float lo = out[t * (hpc * hd) + lh * hd + j];
        const float hi = out[t * (hpc * hd) + lh * hd + j + half];
        const int tok = t0 + t;
        float o1 = lo, o2 = hi;
        if (gh < dm.H + dm.KV) {
            const float angle = __fmul_rn(positions[tok], inv_freq[j]);
            float s, c;
            sincosf(angle, &s, &c);
            c = Store<T>::round(__fmul_rn(c, dm.conc));
            s = Store<T>::round(__fmul_rn(s, dm.conc));
            o1 = Store<T>::round(__fsub_rn(Store<T>::round(__fmul_rn(lo, c)), Store<T>::round(__fmul_rn(hi, s))));
            o2 = Store<T>::round(__fadd_rn(Store<T>::round(__fmul_rn(hi, c)), Store<T>::round(__fmul_rn(lo, s))));
        }
        if (gh < dm.H) {
            float* qrow = q_out + size_t(tok) * dm.H * hd + size_t(gh) * hd;
            qrow[j] = o1;
            qrow[j + half] = o2;
        } else if (gh < dm.H + dm.KV) {
            T* krow = k_out + size_t(tok) * dm.KV * hd + size_t(gh - dm.H) * hd;
            Store<T>::store(krow + j, o1);
            Store<T>::store(krow + j + half, o2);
        } else {
            T* vrow = v_out + size_t(tok) * dm.KV * hd + size_t(gh - dm.H - dm.KV) * hd;
            Store<T>::store(vrow + j, o1);
            Store<T>::store(vrow + j + half, o2);
        }
    }
}

// ------------------------------------------------------------------------------------------------------
// Sink-augmented attention, one CTA per (query row, kv head, sequence), one warp per query head of the group.
// Keys are the `ctx` cache rows followed by the sequence's `n` new rows. Scores are kept in shared memory so the
// probabilities can be rounded like the reference's softmax output before P.V.
struct AttnArgs {
    int n, ctx, B;
    size_t cache_seq_stride;  // elements between sequences in the cache (layer offset already applied)
    int mask_mode;
    int window;               // mask window for kMaskCausal / kMaskSlots (0 = none)
    const int64_t* slots;     // [B][ctx] absolute positions of cache rows (-1 empty)
    const int64_t* pos0;      // [B] absolute position of each sequence's first new row
};

template <typename T>
__global__ void __launch_bounds__(256) k_attention(const float* __restrict__ q, Dims dm, AttnArgs a,
                                                    const T* __restrict__ cache_k, const T* __restrict__ cache_v,
                                                    const T* __restrict__ new_k, const T* __restrict__ new_v,
                                                    const T* __restrict__ bias, const T* __restrict__ sinks,
                                                    float* __restrict__ out) {
    extern __shared__ float scores[];
    const int i = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = dm.hd, nkeys = a.ctx + a.n;
    const int hq = kvh * dm.G + warp;
    const size_t tok = size_t(b) * a.n + i;
    float* sc = scores + size_t(warp) * nkeys;

    pdl_wait();
    pdl_trigger();

    float qv[64];
    const float* qrow = q + tok * dm.H * hd + size_t(hq) * hd;
#pragma unroll
    for (int e = 0; e < 64; ++e)
        if (e < hd) qv[e] = qrow[e];

    const T* ck = cache_k + b * a.cache_seq_stride + size_t(kvh) * hd;
    const T* cv = cache_v + b * a.cache_seq_stride + size_t(kvh) * hd;
    const T* nk = new_k + (size_t(b) * a.n * dm.KV + kvh) * hd;
    const T* nv = new_v + (size_t(b) * a.n * dm.KV + kvh) * hd;
    const size_t kstride = size_t(dm.KV) * hd;

    int64_t t_i = 0;
    if (a.mask_mode == kMaskSlots) t_i = a.pos0[b] + i;

    float mx = -INFINITY;
    for (int j = lane; j < nkeys; j += 32) {
        const T* krow = j < a.ctx ? ck + size_t(j) * kstride : nk + size_t(j - a.ctx) * kstride;
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
            if (e < hd) {
                float k4[4];
                load4(krow + e, k4);
                dot = fmaf(qv[e], k4[0], dot);
                dot = fmaf(qv[e + 1], k4[1], dot);
                dot = fmaf(qv[e + 2], k4[2], dot);
                dot = fmaf(qv[e + 3], k4[3], dot);
            }
        }
        float s = Store<T>::round(__fmul_rn(Store<T>::round(dot), dm.sm_scale));
        if (a.mask_mode == kMaskBuffer) {
            s = Store<T>::round(__fadd_rn(s, Store<T>::load(bias + size_t(i) * nkeys + j)));
        } else {
            bool visible;
            if (a.mask_mode == kMaskCausal) {
                visible = (j - a.ctx) <= i && (a.window <= 0 || i - (j - a.ctx) < a.window);
            } else {
                const int64_t t_j = j < a.ctx ? a.slots[size_t(b) * a.ctx + j] : a.pos0[b] + (j - a.ctx);
                const bool valid = j >= a.ctx || t_j >= 0;
                visible = valid && t_j <= t_i && (a.window <= 0 || t_j > t_i - a.window);
            }
            if (!visible) s = -INFINITY;
        }
        sc[j] = s;
        mx = fmaxf(mx, s);
    }
    const float sink = Store<T>::load(sinks + hq);
    mx = fmaxf(warp_max(mx), sink);
    float l = 0.f;
    for (int j = lane; j < nkeys; j += 32) {
        const float e = expf(sc[j] - mx);
        sc[j] = e;
        l += e;
    }
    l = warp_sum(l) + expf(sink - mx);
    const float rl = l;
    __syncwarp();
    for (int j = lane; j < nkeys; j += 32) sc[j] = Store<T>::round(sc[j] / rl);
    __syncwarp();

    // P.V: lanes split into `groups` key groups of `dl` dims each.
    const int dl = hd < 32 ? hd : 32;
    const int groups = 32 / dl;
    const int g = lane / dl, dd = lane % dl;
    float acc[2] = {0.f, 0.f};
    for (int j = g; j < nkeys; j += groups) {
        const T* vrow = j < a.ctx ? cv + size_t(j) * kstride : nv + size_t(j - a.ctx) * kstride;
        const float p = sc[j];
        acc[0] = fmaf(p, Store<T>::load(vrow + dd), acc[0]);
        if (hd > 32) acc[1] = fmaf(p, Store<T>::load(vrow + dd + 32), acc[1]);
    }
    for (int o = dl; o < 32; o <<= 1) {
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
        acc[1] += __shfl_xor_sync(0xffffffffu, acc[1], o);
    }
    float* orow = out + tok * dm.H * hd + size_t(hq) * hd;
    if (g == 0) {
        orow[dd] = Store<T>::round(acc[0]);
        if (hd > 32) orow[dd + 32] = Store<T>::round(acc[1]);
    }
}

// ------------------------------------------------------------------------------------------------------
// Warp-wide top-k over `n` logits in shared memory: NaN ranks highest, ties go to the lowest index, output
// sorted (the ranking of chroma/_src/codegen/gpu.py:300-337). Then softmax over the k values (kernels.h:125-151).
template <typename T>
__device__ void warp_topk_softmax(const float* g, int n, int k, int* idx_out, float* w_out, int* trace) {
    const int lane = threadIdx.x & 31;
    unsigned taken = 0;  // bit per owned slot (lane + 32*s), n <= 256
    float vals[8];
    int ids[8];
    for (int r = 0; r < k; ++r) {
        float best = 0.f;
        int bi = 0x7fffffff;
        bool have = false;
        for (int s = 0; s < 8; ++s) {
            const int j = lane + 32 * s;
            if (j >= n || (taken >> s & 1u)) continue;
            const float v = g[j];
            bool better;
            if (!have) better = true;
            else if (isnan(v) != isnan(best)) better = isnan(v);
            else better = v > best;
            if (better) { best = v; bi = j; have = true; }
        }
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            bool better;
            if (oi == 0x7fffffff) better = false;
            else if (bi == 0x7fffffff) better = true;
            else if (isnan(ov) != isnan(best)) better = isnan(ov);
            else if (ov != best && !(isnan(ov) && isnan(best))) better = ov > best;
            else better = oi < bi;
            if (better) { best = ov; bi = oi; }
        }
        if ((bi & 31) == lane && bi != 0x7fffffff) taken |= 1u << (bi >> 5);
        vals[r] = best;
        ids[r] = bi;
    }
    if (lane == 0) {
        float m = -INFINITY;
        for (int r = 0; r < k; ++r) m = fmaxf(m, vals[r]);
        float e[8], s = 0.f;
        for (int r = 0; r < k; ++r) { e[r] = expf(vals[r] - m); s += e[r]; }
        for (int r = 0; r < k; ++r) {
            idx_out[r] = ids[r];
            w_out[r] = Store<T>::round(e[r] / s);
            if (trace) trace[r] = ids[r];
        }
    }
}

// grid = ntok; block = 256. Out-projection + residual, then the MLP block's norm, gate and routing. `routes`
// (optional) records this layer's selected experts for inspection.
template <typename T>
__global__ void __launch_bounds__(256) k_out_router(const float* __restrict__ attn, const float* __restrict__ x,
                                                    int ntok, Dims dm, LayerW<T> w, float* __restrict__ x2,
                                                    float* __restrict__ tnorm, int* __restrict__ ridx,
                                                    float* __restrict__ rw, int* __restrict__ routes) {
    extern __shared__ float smem[];
    const int K = dm.H * dm.hd, d = dm.d;
    float* as = smem;       // [K]
    float* xr = as + K;     // [d]
    float* gl = xr + d;     // [E]
    float* red = gl + dm.E; // [32]
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    prefetch_l2(w.out_w, size_t(d) * K * sizeof(T), threadIdx.x, blockDim.x);
    pdl_wait();
    pdl_trigger();

    for (int c = threadIdx.x; c < K; c += blockDim.x) as[c] = attn[size_t(t) * K + c];
    __syncthreads();
    for (int c = warp; c < d; c += warps) {
        float acc[1];
        warp_row_dots<T, 1>(w.out_w + size_t(c) * K, as, K, 1, acc);
        if (lane == 0) {
            const float o = Store<T>::round(__fadd_rn(acc[0], Store<T>::load(w.out_b + c)));
            const float v = Store<T>::round(__fadd_rn(x[size_t(t) * d + c], o));
            xr[c] = v;
            x2[size_t(t) * d + c] = v;
        }
    }
    __syncthreads();
    float s = 0.f;
    for (int c = threadIdx.x; c < d; c += blockDim.x) s = fmaf(xr[c], xr[c], s);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int i = 0; i < warps; ++i) tot += red[i];
        red[0] = 1.0f / sqrtf(tot / float(d) + dm.eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        const float v = Store<T>::round(__fmul_rn(__fmul_rn(xr[c], inv), w.mlp_norm[c]));
        xr[c] = v;
        tnorm[size_t(t) * d + c] = v;
    }
    __syncthreads();
    for (int e = warp; e < dm.E; e += warps) {
        float acc[1];
        warp_row_dots<T, 1>(w.gate_w + size_t(e) * d, xr, d, 1, acc);
        if (lane == 0) gl[e] = Store<T>::round(__fadd_rn(acc[0], Store<T>::load(w.gate_b + e)));
    }
    __syncthreads();
    if (warp == 0)
        warp_topk_softmax<T>(gl, dm.E, dm.k, ridx + size_t(t) * dm.k, rw + size_t(t) * dm.k,
                             routes ? routes + size_t(t) * dm.k : nullptr);
}

// ------------------------------------------------------------------------------------------------------
// grid = (ntok * k, ceil(I / pairs_per_cta)); block = 256. Each warp computes one (glu, linear) row pair of the
// selected expert's mlp1 and applies the clamped SwiGLU (gpt_oss.py:212-219) with the reference's rounding points.
template <typename T>
__global__ void __launch_bounds__(256) k_moe_up(const float* __restrict__ tnorm, int ntok, Dims dm,
                                                const int* __restrict__ ridx, const T* __restrict__ w1,
                                                const T* __restrict__ b1, int pairs_per_cta,
                                                float* __restrict__ act, unsigned* err) {
    extern __shared__ float xs[];  // [d]
    const int te = blockIdx.x;  // token * k + slot
    const int t = te / dm.k;
    const int d = dm.d;
    const int p0 = blockIdx.y * pairs_per_cta;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    const int e = int(checked_row(ridx[te], dm.E, true, err));
    const T* W = w1 + size_t(e) * 2 * dm.I * d;
    const T* B = b1 + size_t(e) * 2 * dm.I;
    for (int c = threadIdx.x; c < d; c += blockDim.x) xs[c] = tnorm[size_t(t) * d + c];
    __syncthreads();
    const int p_end = min(dm.I, p0 + pairs_per_cta);
    for (int p = p0 + warp; p < p_end; p += warps) {
        float ag[1], al[1];
        warp_row_dots<T, 1>(W + size_t(2 * p) * d, xs, d, 1, ag);
        warp_row_dots<T, 1>(W + size_t(2 * p + 1) * d, xs, d, 1, al);
        if (lane == 0) {
            // einsum output (rounded), then + mlp1_bias (rounded) (gpt_oss.py:253).
            const float hg = Store<T>::round(__fadd_rn(Store<T>::round(ag[0]), Store<T>::load(B + 2 * p)));
            const float hl = Store<T>::round(__fadd_rn(Store<T>::round(al[0]), Store<T>::load(B + 2 * p + 1)));
            const float glu = fminf(hg, dm.limit);
            const float lin = fminf(fmaxf(hl, -dm.limit), dm.limit);
            const float z = Store<T>::round(__fmul_rn(glu, dm.alpha));
            const float sg = Store<T>::round(1.0f / (1.0f + expf(-z)));
            const float og = Store<T>::round(__fmul_rn(glu, sg));
            const float l1 = Store<T>::round(__fadd_rn(lin, 1.0f));
            act[size_t(te) * dm.I + p] = Store<T>::round(__fmul_rn(og, l1));
        }
    }
}

// grid = (ntok, ceil(d / cols_per_cta)); block = 256. mlp2 of every selected expert for a slice of output
// columns, + bias, weighted sum over the k experts in slot order, + residual.
template <typename T>
__global__ void __launch_bounds__(256) k_moe_down(const float* __restrict__ act, const float* __restrict__ x2,
                                                  int ntok, Dims dm, const int* __restrict__ ridx,
                                                  const float* __restrict__ rw, const T* __restrict__ w2,
                                                  const T* __restrict__ b2, int cols_per_cta,
                                                  float* __restrict__ x_out, unsigned* err) {
    extern __shared__ float as[];  // [k][I]
    const int t = blockIdx.x;
    const int c0 = blockIdx.y * cols_per_cta;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < dm.k * dm.I; i += blockDim.x) as[i] = act[size_t(t) * dm.k * dm.I + i];
    __syncthreads();
    const int c_end = min(dm.d, c0 + cols_per_cta);
    for (int c = c0 + warp; c < c_end; c += warps) {
        float comb = 0.f;
        for (int s = 0; s < dm.k; ++s) {
            const int e = int(checked_row(ridx[size_t(t) * dm.k + s], dm.E, true, err));
            float acc[1];
            warp_row_dots<T, 1>(w2 + (size_t(e) * dm.d + c) * dm.I, as + s * dm.I, dm.I, 1, acc);
            const float y = Store<T>::round(__fadd_rn(Store<T>::round(acc[0]), Store<T>::load(b2 + size_t(e) * dm.d + c)));
            comb = __fadd_rn(comb, __fmul_rn(y, rw[size_t(t) * dm.k + s]));
        }
        if (lane == 0) {
            const float cm = Store<T>::round(comb);
            x_out[size_t(t) * dm.d + c] = Store<T>::round(__fadd_rn(x2[size_t(t) * dm.d + c], cm));
        }
    }
}

// ------------------------------------------------------------------------------------------------------
// Final RMSNorm of selected rows: rows[r] = index of the r-th wanted row (negative wraps, aten.index semantics).
template <typename T>
__global__ void k_final_norm(const float* __restrict__ x, int ntok, int nrows, const int64_t* __restrict__ rows,
                             int rows_per_seq, const float* __restrict__ norm_w, Dims dm, float* __restrict__ out,
                             unsigned* err) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    int64_t src = r;
    if (rows != nullptr) {
        // One selected row per sequence; rows[] holds the row index within each sequence.
        const int seq = r;
        src = int64_t(seq) * rows_per_seq + checked_row(rows[seq], rows_per_seq, true, err);
    }
    const float* xr = x + size_t(src) * dm.d;
    float s = 0.f;
    for (int c = threadIdx.x; c < dm.d; c += blockDim.x) s = fmaf(xr[c], xr[c], s);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        float tot = 0.f;
        for (int i = 0; i < warps; ++i) tot += red[i];
        red[0] = 1.0f / sqrtf(tot / float(dm.d) + dm.eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int c = threadIdx.x; c < dm.d; c += blockDim.x)
        out[size_t(r) * dm.d + c] = Store<T>::round(__fmul_rn(__fmul_rn(xr[c], inv), norm_w[c]));
}

// Vocab projection: logits[r][v] = sum_c xs[r][c] * W[v][c], rows R <= 8 per pass. Each warp covers 4 vocab rows per
// step with 8 lanes per row; the grid strides over blocks of rows. Weights stream once (no L1 allocation).
constexpr int kVocabRows = 8;

template <typename T, int R>
__global__ void __launch_bounds__(256) k_vocab(const float* __restrict__ xin, int nrows, int d, int V,
                                               const T* __restrict__ W, T* __restrict__ logits) {
    extern __shared__ float xs[];  // [R][d]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane & 7, grp = lane >> 3;
    const int warps_total = gridDim.x * (blockDim.x >> 5);
    const int gw = blockIdx.x * (blockDim.x >> 5) + warp;
    pdl_wait();
    pdl_trigger();
    for (int r0 = 0; r0 < nrows; r0 += R) {
        const int rr = min(R, nrows - r0);
        __syncthreads();
        for (int i = threadIdx.x; i < rr * d; i += blockDim.x) xs[i] = xin[size_t(r0) * d + i];
        __syncthreads();
        for (int v0 = gw * 4; v0 < V; v0 += warps_total * 4) {
            const int v = v0 + grp;
            float acc[R];
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
            if (v < V) {
                const T* wrow = W + size_t(v) * d;
                for (int c = sub * 4; c < d; c += 32) {
                    float w4[4];
                    load4_stream(wrow + c, w4);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        if (r < rr) {
                            const float4 xv = *reinterpret_cast<const float4*>(xs + r * d + c);
                            acc[r] = fmaf(w4[0], xv.x, acc[r]);
                            acc[r] = fmaf(w4[1], xv.y, acc[r]);
                            acc[r] = fmaf(w4[2], xv.z, acc[r]);
                            acc[r] = fmaf(w4[3], xv.w, acc[r]);
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = group_sum(acc[r], 8);
            if (sub == 0 && v < V) {
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (r < rr) Store<T>::store(logits + size_t(r0 + r) * V + v, acc[r]);
            }
        }
    }
}

}  // namespace cb200
