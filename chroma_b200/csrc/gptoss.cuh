// GPT-OSS-style transformer kernels (fp32 or bf16 storage) for token counts up to a few hundred per launch
// (decode steps, prefill chunks, short forwards).
//
// One fused kernel per stage of the block, replacing the reference's chain of generated one-thread-per-element
// kernels plus cuBLAS calls (chroma/_src/codegen/gpu.py:165-424, chroma/_src/codegen/cuda/codegen.py:87-140):
//
//   k_embed         embedding gather with bounds check                          (gpt_oss.py:304-306)
//   k_attn_in       RMSNorm -> QKV linear (+bias) -> RoPE -> q, new K/V rows    (gpt_oss.py:189-202)
//   k_attention     scores*scale + mask, sink column, softmax, P.V, split over key chunks
//                                                                                (gpt_oss.py:133-151, cached.py:36-47)
//   k_out           out linear (+bias) + residual                               (gpt_oss.py:204-209)
//   k_moe_up        RMSNorm -> gate -> top-k -> softmax, then the selected expert's mlp1 (+bias) -> SwiGLU
//                                                                                (gpt_oss.py:243-254, 212-219)
//   k_moe_down      selected experts' mlp2 (+bias) -> weighted combine -> residual (gpt_oss.py:257-265)
//   k_final_norm    final RMSNorm of the rows whose logits are wanted            (gpt_oss.py:309, cached.py:50)
//   k_vocab         unembedding GEMV with a fused greedy argmax                  (gpt_oss.py:310)
//
// Decode-sized work is latency-bound, so every GEMV is written for memory-level parallelism: a warp owns a few
// weight rows, each lane issues all of its 16-byte loads for those rows before any arithmetic, and the first chunk
// of weights is loaded BEFORE the programmatic-dependent-launch wait, overlapping the previous kernel's tail.
//
// Activations live in fp32 buffers; for bf16 programs every value is rounded to bf16 wherever the exported graph
// rounds it (after each linear, einsum, residual add and SwiGLU step), so results track the reference's CPU program.
#pragma once

#include "common.cuh"
#include "tma.cuh"

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

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTileTokens = 8;  // activation rows per CTA tile in the GEMV kernels
constexpr int kMJ = 4;          // float4 chunks per lane per row in one fragment: 512 elements per chunk pass
constexpr int kChunk = 128 * kMJ;

// ------------------------------------------------------------------------------------------------------
// Register fragment of up to MR weight rows: lane l holds elements c0 + 4*l + 128*j (j < kMJ) of each row.
template <int MR> struct Frag {
    float v[MR][kMJ][4];
};

template <typename T, int MR>
__device__ __forceinline__ void frag_load(Frag<MR>& f, const T* const (&rows)[MR], int nr, int d, int c0) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int r = 0; r < MR; ++r)
#pragma unroll
        for (int j = 0; j < kMJ; ++j) {
            const int c = c0 + lane * 4 + 128 * j;
            if (r < nr && c < d) {
                load4(rows[r] + c, f.v[r][j]);
            } else {
                f.v[r][j][0] = f.v[r][j][1] = f.v[r][j][2] = f.v[r][j][3] = 0.f;
            }
        }
}

// acc[r][t] += frag row r . xs row t over the fragment's chunk (xs: fp32 rows of stride d in shared memory).
template <int MR, int TT>
__device__ __forceinline__ void frag_fma(const Frag<MR>& f, const float* xs, int d, int tt, int c0, float (&acc)[MR][TT]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < kMJ; ++j) {
        const int c = c0 + lane * 4 + 128 * j;
        if (c < d) {
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                if (t < tt) {
                    const float4 x = *reinterpret_cast<const float4*>(xs + t * d + c);
#pragma unroll
                    for (int r = 0; r < MR; ++r) {
                        acc[r][t] = fmaf(f.v[r][j][0], x.x, acc[r][t]);
                        acc[r][t] = fmaf(f.v[r][j][1], x.y, acc[r][t]);
                        acc[r][t] = fmaf(f.v[r][j][2], x.z, acc[r][t]);
                        acc[r][t] = fmaf(f.v[r][j][3], x.w, acc[r][t]);
                    }
                }
            }
        }
    }
}

// Full dot products of MR rows with tt activation rows; `f` must already hold the chunk at c0 = 0.
template <typename T, int MR, int TT>
__device__ __forceinline__ void warp_gemv(Frag<MR>& f, const T* const (&rows)[MR], int nr, const float* xs, int d, int tt,
                                          float (&acc)[MR][TT]) {
#pragma unroll
    for (int r = 0; r < MR; ++r)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[r][t] = 0.f;
    for (int c0 = 0;;) {
        frag_fma<MR, TT>(f, xs, d, tt, c0, acc);
        c0 += kChunk;
        if (c0 >= d) break;
        frag_load<T, MR>(f, rows, nr, d, c0);
    }
#pragma unroll
    for (int r = 0; r < MR; ++r)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[r][t] = warp_sum(acc[r][t]);
}

// Normalise `tt` rows staged in shared memory in place: x * (1/sqrt(mean(x^2) + eps)) * w, rounded to storage
// (the fused norm of chroma/_src/codegen/cpu/kernels.h:101-115). `inv` is [tt] scratch.
template <typename T>
__device__ __forceinline__ void rows_rmsnorm(float* xs, int tt, int d, float eps, const float* __restrict__ w, float* inv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int r = warp; r < tt; r += warps) {
        float s = 0.f;
        for (int c = lane; c < d; c += 32) s = fmaf(xs[r * d + c], xs[r * d + c], s);
        s = warp_sum(s);
        if (lane == 0) inv[r] = 1.0f / sqrtf(s / float(d) + eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < tt * d; i += blockDim.x)
        xs[i] = Store<T>::round(__fmul_rn(__fmul_rn(xs[i], inv[i / d]), w[i % d]));
    __syncthreads();
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
// grid = (heads_total, ceil(ntok / kTileTokens)); block = kThreads. A CTA owns one head of the fused QKV projection
// (so both halves of each RoPE pair are local); each warp owns 2 of its rows at a time.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_attn_in(const float* __restrict__ x, int ntok, Dims dm,
                                                      const float* __restrict__ norm_w, const T* __restrict__ W,
                                                      const T* __restrict__ bias, const float* __restrict__ positions,
                                                      const float* __restrict__ inv_freq, float* __restrict__ q_out,
                                                      T* __restrict__ k_out, T* __restrict__ v_out) {
    extern __shared__ float smem[];
    constexpr int TT = kTileTokens, MR = 2;
    const int d = dm.d, hd = dm.hd;
    const int head = blockIdx.x;
    const int t0 = blockIdx.y * TT;
    const int tt = min(TT, ntok - t0);
    float* xs = smem;            // [TT][d]
    float* out = xs + TT * d;    // [TT][hd]
    float* inv = out + TT * hd;  // [TT]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int r0 = warp * MR;
    const T* rows[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) rows[r] = W + size_t(head * hd + min(r0 + r, hd - 1)) * d;
    Frag<MR> f;
    frag_load<T, MR>(f, rows, max(0, min(MR, hd - r0)), d, 0);
    pdl_wait();
    pdl_trigger();

    for (int i = threadIdx.x; i < tt * d; i += blockDim.x) xs[i] = x[size_t(t0) * d + i];
    __syncthreads();
    rows_rmsnorm<T>(xs, tt, d, dm.eps, norm_w, inv);

    for (int rb = r0; rb < hd; rb += kWarps * MR) {
        const int nr = min(MR, hd - rb);
        if (rb != r0) {
#pragma unroll
            for (int r = 0; r < MR; ++r) rows[r] = W + size_t(head * hd + min(rb + r, hd - 1)) * d;
            frag_load<T, MR>(f, rows, nr, d, 0);
        }
        float acc[MR][TT];
        warp_gemv<T, MR, TT>(f, rows, nr, xs, d, tt, acc);
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                if (r >= nr) break;
                const float b = Store<T>::load(bias + head * hd + rb + r);
#pragma unroll
                for (int t = 0; t < TT; ++t)
                    if (t < tt) out[t * hd + rb + r] = Store<T>::round(__fadd_rn(acc[r][t], b));
            }
        }
    }
    __syncthreads();

    // RoPE on q and k heads (gpt_oss.py:44-54): o1 = x1*cos - x2*sin, o2 = x2*cos + x1*sin, cos/sin rounded to
    // storage first; v heads pass through.
    const int half = hd / 2;
    for (int i = threadIdx.x; i < tt * half; i += blockDim.x) {
        const int t = i / half, j = i % half;
        const float lo = out[t * hd + j];
        const float hi = out[t * hd + j + half];
        const int tok = t0 + t;
        float o1 = lo, o2 = hi;
        if (head < dm.H + dm.KV) {
            const float angle = __fmul_rn(positions[tok], inv_freq[j]);
            float s, c;
            sincosf(angle, &s, &c);
            c = Store<T>::round(__fmul_rn(c, dm.conc));
            s = Store<T>::round(__fmul_rn(s, dm.conc));
            o1 = Store<T>::round(__fsub_rn(Store<T>::round(__fmul_rn(lo, c)), Store<T>::round(__fmul_rn(hi, s))));
            o2 = Store<T>::round(__fadd_rn(Store<T>::round(__fmul_rn(hi, c)), Store<T>::round(__fmul_rn(lo, s))));
        }
        if (head < dm.H) {
            float* qrow = q_out + size_t(tok) * dm.H * hd + size_t(head) * hd;
            qrow[j] = o1;
            qrow[j + half] = o2;
        } else {
            T* dst = head < dm.H + dm.KV ? k_out + size_t(tok) * dm.KV * hd + size_t(head - dm.H) * hd
                                         : v_out + size_t(tok) * dm.KV * hd + size_t(head - dm.H - dm.KV) * hd;
            Store<T>::store(dst + j, o1);
            Store<T>::store(dst + j + half, o2);
        }
    }
}

// ------------------------------------------------------------------------------------------------------
// Sink-augmented attention over key chunks. grid = (query row, kv head, sequence * chunks); block = kThreads.
// Each CTA stages one chunk of K and V rows in shared memory (cache rows before the PDL wait: no kernel of the
// running step writes them), scores it for the G query heads of its kv head (one warp each), and either finishes
// the softmax directly (single chunk: probabilities rounded like the reference's softmax output) or writes an
// (m, l, o) partial that the last CTA of the row merges with the sink logit (split-KV, flash-decoding style).
struct AttnArgs {
    int n, ctx, B, chunks, key_chunk;  // key_chunk: keys per CTA (512 for head_dim <= 32, else 256)
    size_t cache_seq_stride;  // elements between sequences in the cache (layer offset already applied)
    int mask_mode;
    int window;               // mask window for kMaskCausal / kMaskSlots (0 = none)
    const int64_t* slots;     // [B][ctx] absolute positions of cache rows (-1 empty)
    const int64_t* pos0;      // [B] absolute position of each sequence's first new row
    float* partial;           // [B*n][KV][G][chunks][hd + 2] split-KV partials
    unsigned* counters;       // [B*n][KV] arrival counters, left at zero
};

template <typename T, typename TQ = float>
__global__ void __launch_bounds__(kThreads) k_attention(const TQ* __restrict__ q, Dims dm, AttnArgs a,
                                                        const T* __restrict__ cache_k, const T* __restrict__ cache_v,
                                                        const T* __restrict__ new_k, const T* __restrict__ new_v,
                                                        const T* __restrict__ bias, const T* __restrict__ sinks,
                                                        TQ* __restrict__ out) {
    extern __shared__ float sm[];
    const int i = blockIdx.x, kvh = blockIdx.y;
    const int b = blockIdx.z / a.chunks, chunk = blockIdx.z % a.chunks;
    const int hd = dm.hd, G = dm.G, stride = hd + 1;
    const int nkeys = a.ctx + a.n;
    const int KC = a.key_chunk;
    const int j0 = chunk * KC;
    const int nk = min(KC, nkeys - j0);
    float* Ks = sm;                   // [KC][hd+1]
    float* Vs = Ks + KC * stride;     // [KC][hd+1]
    float* sc = Vs + KC * stride;     // [G][KC]
    float* qs = sc + G * KC;          // [G][hd]
    __shared__ unsigned last_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const size_t tok = size_t(b) * a.n + i;
    const size_t kstride = size_t(dm.KV) * hd;
    const int q4 = hd / 4;

    const T* ck = cache_k + b * a.cache_seq_stride + size_t(kvh) * hd;
    const T* cv = cache_v + b * a.cache_seq_stride + size_t(kvh) * hd;
    const T* nkp = new_k + (size_t(b) * a.n * dm.KV + kvh) * hd;
    const T* nvp = new_v + (size_t(b) * a.n * dm.KV + kvh) * hd;
    // Cache rows of this chunk.
    for (int e = threadIdx.x; e < nk * q4; e += blockDim.x) {
        const int jj = e / q4, c = (e % q4) * 4, j = j0 + jj;
        if (j < a.ctx) {
            float kv[4], vv[4];
            load4(ck + size_t(j) * kstride + c, kv);
            load4(cv + size_t(j) * kstride + c, vv);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                Ks[jj * stride + c + u] = kv[u];
                Vs[jj * stride + c + u] = vv[u];
            }
        }
    }
    pdl_wait();
    pdl_trigger();
    for (int e = threadIdx.x; e < nk * q4; e += blockDim.x) {
        const int jj = e / q4, c = (e % q4) * 4, j = j0 + jj;
        if (j >= a.ctx) {
            float kv[4], vv[4];
            load4(nkp + size_t(j - a.ctx) * kstride + c, kv);
            load4(nvp + size_t(j - a.ctx) * kstride + c, vv);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                Ks[jj * stride + c + u] = kv[u];
                Vs[jj * stride + c + u] = vv[u];
            }
        }
    }
    for (int e = threadIdx.x; e < G * hd; e += blockDim.x)
        qs[e] = Store<TQ>::load(q + tok * dm.H * hd + size_t(kvh) * G * hd + e);
    __syncthreads();

    int64_t t_i = 0;
    if (a.mask_mode == kMaskSlots) t_i = a.pos0[b] + i;
    const int dl = hd < 32 ? hd : 32;
    const int groups = 32 / dl;
    const int g = lane / dl, dd = lane % dl;

    for (int m = warp; m < G; m += kWarps) {
        const int hq = kvh * G + m;
        const float* qv = qs + m * hd;
        float* s_row = sc + m * KC;
        float mx = -INFINITY;
        for (int jj = lane; jj < nk; jj += 32) {
            const int j = j0 + jj;
            const float* kr = Ks + jj * stride;
            float dot = 0.f;
            for (int e = 0; e < hd; ++e) dot = fmaf(qv[e], kr[e], dot);
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
            s_row[jj] = s;
            mx = fmaxf(mx, s);
        }
        mx = warp_max(mx);
        const float sink = Store<T>::load(sinks + hq);
        const bool single = a.chunks == 1;
        // Single chunk: normalise against max(m, sink) now; otherwise keep chunk-local (m, l) for the merge.
        const float ref = single ? fmaxf(mx, sink) : mx;
        float l = 0.f;
        for (int jj = lane; jj < nk; jj += 32) {
            const float p = ref == -INFINITY ? 0.f : expf(s_row[jj] - ref);
            s_row[jj] = p;
            l += p;
        }
        l = warp_sum(l);
        if (single) {
            l += expf(sink - ref);
            __syncwarp();
            for (int jj = lane; jj < nk; jj += 32) s_row[jj] = Store<T>::round(s_row[jj] / l);
        }
        __syncwarp();
        float acc[2] = {0.f, 0.f};
        for (int jj = g; jj < nk; jj += groups) {
            const float p = s_row[jj];
            acc[0] = fmaf(p, Vs[jj * stride + dd], acc[0]);
            if (hd > 32) acc[1] = fmaf(p, Vs[jj * stride + dd + 32], acc[1]);
        }
        for (int o = dl; o < 32; o <<= 1) {
            acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
            acc[1] += __shfl_xor_sync(0xffffffffu, acc[1], o);
        }
        if (single) {
            TQ* orow = out + tok * dm.H * hd + size_t(hq) * hd;
            if (g == 0) {
                Store<TQ>::store(orow + dd, Store<T>::round(acc[0]));
                if (hd > 32) Store<TQ>::store(orow + dd + 32, Store<T>::round(acc[1]));
            }
        } else {
            float* part = a.partial + (((tok * dm.KV + kvh) * G + m) * a.chunks + chunk) * (hd + 2);
            if (g == 0) {
                part[2 + dd] = acc[0];
                if (hd > 32) part[2 + dd + 32] = acc[1];
            }
            if (lane == 0) {
                part[0] = mx;
                part[1] = l;
            }
        }
    }
    if (a.chunks == 1) return;
    // Split-KV merge: the last CTA of this (row, kv head) combines every chunk's partial with the sink.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.counters + tok * dm.KV + kvh, 1u);
        last_flag = prev == unsigned(a.chunks - 1);
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    for (int m = warp; m < G; m += kWarps) {
        const int hq = kvh * G + m;
        const float* part = a.partial + ((tok * dm.KV + kvh) * G + m) * a.chunks * (hd + 2);
        const float sink = Store<T>::load(sinks + hq);
        float M = sink;
        for (int c = 0; c < a.chunks; ++c) M = fmaxf(M, part[c * (hd + 2)]);
        float L = expf(sink - M);
        for (int c = 0; c < a.chunks; ++c) {
            const float mc = part[c * (hd + 2)];
            if (mc != -INFINITY) L += part[c * (hd + 2) + 1] * expf(mc - M);
        }
        TQ* orow = out + tok * dm.H * hd + size_t(hq) * hd;
        for (int e = lane; e < hd; e += 32) {
            float o = 0.f;
            for (int c = 0; c < a.chunks; ++c) {
                const float mc = part[c * (hd + 2)];
                if (mc != -INFINITY) o += part[c * (hd + 2) + 2 + e] * expf(mc - M);
            }
            Store<TQ>::store(orow + e, Store<T>::round(o / L));
        }
    }
    if (threadIdx.x == 0) a.counters[tok * dm.KV + kvh] = 0u;
}

// ------------------------------------------------------------------------------------------------------
// grid = (ceil(d / (kWarps*2)), ceil(ntok / kTileTokens)); block = kThreads. Out-projection + bias + residual.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_out(const float* __restrict__ attn, const float* __restrict__ x, int ntok,
                                                  Dims dm, const T* __restrict__ Wo, const T* __restrict__ bo,
                                                  float* __restrict__ x2) {
    extern __shared__ float as[];  // [TT][K]
    constexpr int TT = kTileTokens, MR = 2;
    const int K = dm.H * dm.hd, d = dm.d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * kWarps * MR + warp * MR;
    const int t0 = blockIdx.y * TT, tt = min(TT, ntok - t0);
    const int nr = max(0, min(MR, d - r0));
    const T* rows[MR];
#pragma unroll
    for (int r = 0; r < MR; ++r) rows[r] = Wo + size_t(min(r0 + r, d - 1)) * K;
    Frag<MR> f;
    frag_load<T, MR>(f, rows, nr, K, 0);
    pdl_wait();
    pdl_trigger();
    for (int e = threadIdx.x; e < tt * K; e += blockDim.x) as[e] = attn[size_t(t0) * K + e];
    __syncthreads();
    if (nr == 0) return;
    float acc[MR][TT];
    warp_gemv<T, MR, TT>(f, rows, nr, as, K, tt, acc);
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < MR; ++r) {
            if (r >= nr) break;
            const float b = Store<T>::load(bo + r0 + r);
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                if (t >= tt) break;
                const size_t o = size_t(t0 + t) * d + r0 + r;
                x2[o] = Store<T>::round(__fadd_rn(x[o], Store<T>::round(__fadd_rn(acc[r][t], b))));
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------------
// Warp-wide top-k over `n` logits in shared memory: NaN ranks highest, ties go to the lowest index, output
// sorted (the ranking of chroma/_src/codegen/gpu.py:300-337). Then softmax over the k values (kernels.h:125-151).
template <typename T>
__device__ void warp_topk_softmax(const float* g, int n, int k, int* idx_out, float* w_out) {
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
        }
    }
}

// grid = (ntok * k, ceil(I / kPairsPerCta)); block = kThreads. Every CTA recomputes its token's router (norm, gate,
// top-k, softmax: a few KB of L2-resident weights) so no separate router launch is needed; the (slot 0, block 0) CTA
// publishes the routing for k_moe_down and for inspection. Then each warp computes 2 (glu, linear) row pairs of the
// CTA's expert and applies the clamped SwiGLU (gpt_oss.py:212-219) with the reference's rounding points.
constexpr int kPairsPerCta = kWarps * 2;

template <typename T>
__global__ void __launch_bounds__(kThreads) k_moe_up(const float* __restrict__ x2, int ntok, Dims dm, LayerW<T> w,
                                                     int* __restrict__ ridx, float* __restrict__ rw,
                                                     int* __restrict__ routes, float* __restrict__ act, unsigned* err) {
    extern __shared__ float sm[];
    const int d = dm.d;
    float* xs = sm;            // [d]
    float* gl = xs + d;        // [E]
    float* misc = gl + dm.E;   // [1 + 8 + 8]: inv, indices, weights
    int* sidx = reinterpret_cast<int*>(misc + 1);
    float* sw = misc + 9;
    const int te = blockIdx.x;  // token * k + slot
    const int t = te / dm.k, slot = te % dm.k;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    for (int c = threadIdx.x; c < d; c += blockDim.x) xs[c] = x2[size_t(t) * d + c];
    __syncthreads();
    rows_rmsnorm<T>(xs, 1, d, dm.eps, w.mlp_norm, misc);
    // Gate: rows e of gate_w, two per warp at a time.
    for (int e0 = warp * 2; e0 < dm.E; e0 += kWarps * 2) {
        const T* rows[2] = {w.gate_w + size_t(e0) * d, w.gate_w + size_t(min(e0 + 1, dm.E - 1)) * d};
        const int nr = min(2, dm.E - e0);
        Frag<2> f;
        frag_load<T, 2>(f, rows, nr, d, 0);
        float acc[2][1];
        warp_gemv<T, 2, 1>(f, rows, nr, xs, d, 1, acc);
        if (lane == 0) {
            gl[e0] = Store<T>::round(__fadd_rn(acc[0][0], Store<T>::load(w.gate_b + e0)));
            if (nr > 1) gl[e0 + 1] = Store<T>::round(__fadd_rn(acc[1][0], Store<T>::load(w.gate_b + e0 + 1)));
        }
    }
    __syncthreads();
    if (warp == 0) warp_topk_softmax<T>(gl, dm.E, dm.k, sidx, sw);
    __syncthreads();
    if (slot == 0 && blockIdx.y == 0 && threadIdx.x < dm.k) {
        ridx[size_t(t) * dm.k + threadIdx.x] = sidx[threadIdx.x];
        rw[size_t(t) * dm.k + threadIdx.x] = sw[threadIdx.x];
        if (routes) routes[size_t(t) * dm.k + threadIdx.x] = sidx[threadIdx.x];
    }
    const int e = int(checked_row(sidx[slot], dm.E, true, err));
    const T* W = w.w1 + size_t(e) * 2 * dm.I * d;
    const T* B = w.b1 + size_t(e) * 2 * dm.I;
    const int p = blockIdx.y * kPairsPerCta + warp * 2;  // this warp's first pair
    if (p >= dm.I) return;
    const int np = min(2, dm.I - p);
    const int p1 = min(p + 1, dm.I - 1);
    const T* rows[4] = {W + size_t(2 * p) * d, W + size_t(2 * p + 1) * d, W + size_t(2 * p1) * d, W + size_t(2 * p1 + 1) * d};
    Frag<4> f;
    frag_load<T, 4>(f, rows, 2 * np, d, 0);
    float acc[4][1];
    warp_gemv<T, 4, 1>(f, rows, 2 * np, xs, d, 1, acc);
    if (lane < np) {
        const int pp = p + lane;
        const float ag = lane == 0 ? acc[0][0] : acc[2][0];
        const float al = lane == 0 ? acc[1][0] : acc[3][0];
        // einsum output (rounded), then + mlp1_bias (rounded) (gpt_oss.py:253).
        const float hg = Store<T>::round(__fadd_rn(Store<T>::round(ag), Store<T>::load(B + 2 * pp)));
        const float hl = Store<T>::round(__fadd_rn(Store<T>::round(al), Store<T>::load(B + 2 * pp + 1)));
        const float glu = fminf(hg, dm.limit);
        const float lin = fminf(fmaxf(hl, -dm.limit), dm.limit);
        const float z = Store<T>::round(__fmul_rn(glu, dm.alpha));
        const float sg = Store<T>::round(1.0f / (1.0f + expf(-z)));
        const float og = Store<T>::round(__fmul_rn(glu, sg));
        const float l1 = Store<T>::round(__fadd_rn(lin, 1.0f));
        act[size_t(te) * dm.I + pp] = Store<T>::round(__fmul_rn(og, l1));
    }
}

// grid = (ntok, ceil(d / kWarps)); block = kThreads. One output column per warp: mlp2 row of each selected expert
// (+ bias), weighted sum over the k experts in slot order, + residual. The k rows are loaded together.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_moe_down(const float* __restrict__ act, const float* __restrict__ x2,
                                                       int ntok, Dims dm, const int* __restrict__ ridx,
                                                       const float* __restrict__ rw, const T* __restrict__ w2,
                                                       const T* __restrict__ b2, float* __restrict__ x_out,
                                                       unsigned* err) {
    extern __shared__ float as[];  // [k][I]
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.y * kWarps + warp;
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < dm.k * dm.I; i += blockDim.x) as[i] = act[size_t(t) * dm.k * dm.I + i];
    __syncthreads();
    if (c >= dm.d) return;
    float comb = 0.f;
    for (int s0 = 0; s0 < dm.k; s0 += 4) {
        const int ns = min(4, dm.k - s0);
        int e[4];
        const T* rows[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            e[u] = int(checked_row(ridx[size_t(t) * dm.k + min(s0 + u, dm.k - 1)], dm.E, true, err));
            rows[u] = w2 + (size_t(e[u]) * dm.d + c) * dm.I;
        }
        // All (up to 4) rows in flight at once; each is then dotted with its own expert's activation row.
        float part[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c0 = 0; c0 < dm.I; c0 += kChunk) {
            Frag<4> f;
            frag_load<T, 4>(f, rows, ns, dm.I, c0);
#pragma unroll
            for (int j = 0; j < kMJ; ++j) {
                const int cc = c0 + lane * 4 + 128 * j;
                if (cc >= dm.I) break;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (u >= ns) break;
                    const float4 xv = *reinterpret_cast<const float4*>(as + (s0 + u) * dm.I + cc);
                    part[u] = fmaf(f.v[u][j][0], xv.x, part[u]);
                    part[u] = fmaf(f.v[u][j][1], xv.y, part[u]);
                    part[u] = fmaf(f.v[u][j][2], xv.z, part[u]);
                    part[u] = fmaf(f.v[u][j][3], xv.w, part[u]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) part[u] = warp_sum(part[u]);
        for (int u = 0; u < ns; ++u) {
            const float y = Store<T>::round(__fadd_rn(Store<T>::round(part[u]), Store<T>::load(b2 + size_t(e[u]) * dm.d + c)));
            comb = __fadd_rn(comb, __fmul_rn(y, rw[size_t(t) * dm.k + s0 + u]));
        }
    }
    if (lane == 0) {
        const float cm = Store<T>::round(comb);
        x_out[size_t(t) * dm.d + c] = Store<T>::round(__fadd_rn(x2[size_t(t) * dm.d + c], cm));
    }
}

// ------------------------------------------------------------------------------------------------------
// Final RMSNorm of selected rows: rows[s] = row within sequence s (negative wraps, aten.index semantics), or every
// row when rows == nullptr. Also clears the argmax keys the vocab kernel accumulates into.
template <typename T>
__global__ void k_final_norm(const float* __restrict__ x, int nrows, const int64_t* __restrict__ rows, int rows_per_seq,
                             const float* __restrict__ norm_w, Dims dm, float* __restrict__ out,
                             unsigned long long* __restrict__ keys, unsigned* err) {
    __shared__ float red[32];
    const int r = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    int64_t src = r;
    if (rows != nullptr) src = int64_t(r) * rows_per_seq + checked_row(rows[r], rows_per_seq, true, err);
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
        if (keys) keys[r] = 0ull;
    }
    __syncthreads();
    const float inv = red[0];
    for (int c = threadIdx.x; c < dm.d; c += blockDim.x)
        out[size_t(r) * dm.d + c] = Store<T>::round(__fmul_rn(__fmul_rn(xr[c], inv), norm_w[c]));
}

// Vocab projection: logits[r][v] = sum_c xs[r][c] * W[v][c] for up to R rows per pass. 8 lanes per vocab row, 4 rows
// per warp step, U steps unrolled (4 for a single activation row, 2 otherwise): every lane issues its 16-byte
// streaming loads for 4*U vocab rows before any FMA. With `keys`, each row's greedy argmax is reduced in-block and merged with one 64-bit atomicMax per block.
constexpr int kVocabRows = 8;

template <typename T, int R>
__global__ void __launch_bounds__(kThreads) k_vocab(const float* __restrict__ xin, int nrows, int d, int V,
                                                    const T* __restrict__ W, T* __restrict__ logits,
                                                    unsigned long long* __restrict__ keys) {
    extern __shared__ float xs[];  // [R][d]
    __shared__ unsigned long long best_s[kWarps][R];
    constexpr int U = R == 1 ? 4 : 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane & 7, grp = lane >> 3;
    const int warps_total = gridDim.x * kWarps;
    const int gw = blockIdx.x * kWarps + warp;
    const int jn = (d + 31) / 32;  // float4 per lane per row
    pdl_wait();
    pdl_trigger();
    for (int r0 = 0; r0 < nrows; r0 += R) {
        const int rr = min(R, nrows - r0);
        __syncthreads();
        for (int i = threadIdx.x; i < rr * d; i += blockDim.x) xs[i] = xin[size_t(r0) * d + i];
        __syncthreads();
        unsigned long long best[R];
#pragma unroll
        for (int r = 0; r < R; ++r) best[r] = 0ull;
        for (int v0 = gw * 4 * U; v0 < V; v0 += warps_total * 4 * U) {
            float acc[U][R];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int r = 0; r < R; ++r) acc[u][r] = 0.f;
            for (int jb = 0; jb < jn; jb += 4) {
                float w[U][4][4];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int v = v0 + u * 4 + grp;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int c = (jb + j) * 32 + sub * 4;
                        if (v < V && jb + j < jn && c < d) load4_stream(W + size_t(v) * d + c, w[u][j]);
                        else w[u][j][0] = w[u][j][1] = w[u][j][2] = w[u][j][3] = 0.f;
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (jb + j >= jn) break;
                    const int c = (jb + j) * 32 + sub * 4;
                    if (c >= d) continue;
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        if (r >= rr) break;
                        const float4 x = *reinterpret_cast<const float4*>(xs + r * d + c);
#pragma unroll
                        for (int u = 0; u < U; ++u) {
                            acc[u][r] = fmaf(w[u][j][0], x.x, acc[u][r]);
                            acc[u][r] = fmaf(w[u][j][1], x.y, acc[u][r]);
                            acc[u][r] = fmaf(w[u][j][2], x.z, acc[u][r]);
                            acc[u][r] = fmaf(w[u][j][3], x.w, acc[u][r]);
                        }
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int v = v0 + u * 4 + grp;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float val = Store<T>::round(group_sum(acc[u][r], 8));
                    if (sub == 0 && v < V && r < rr) {
                        if (logits) Store<T>::store(logits + size_t(r0 + r) * V + v, val);
                        best[r] = max(best[r], argmax_key(val, v));
                    }
                }
            }
        }
        if (keys) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                unsigned long long b = best[r];
                for (int o = 16; o; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
                if (lane == 0) best_s[warp][r] = b;
            }
            __syncthreads();
            if (threadIdx.x < rr) {
                unsigned long long b = 0ull;
                for (int w = 0; w < kWarps; ++w) b = max(b, best_s[w][threadIdx.x]);
                atomicMax(keys + r0 + threadIdx.x, b);
            }
        }
    }
}

// Vocab projection of ONE fp32 activation row (decode steps) with d = 128: the CTA owns a contiguous, balanced range
// of vocab rows (a multiple of 8), so every SM streams the same number of bytes; 8 lanes per vocab row, 4 rows per
// warp step, 2 steps unrolled (16-byte streaming loads of 8 rows in flight per lane); the activation row lives in
// registers. The first step's weights are requested before the programmatic-dependent-launch wait (weights never
// depend on the previous kernel). Same arithmetic and order as k_vocab<float, 1> (per-lane FMA chain, 8-lane butterfly),
// hence the same bits. Measured on B200 at 23.3 us for the 103 MB dev vocab, the time a plain streaming read of the
// same bytes takes (k_vocab<float, 1>: 25.4 us).
constexpr int kVrThreads = 512, kVrU = 2;

__global__ void __launch_bounds__(kVrThreads) k_vocab_row(const float* __restrict__ xin, int V, const float* __restrict__ W,
                                                          float* __restrict__ logits, unsigned long long* __restrict__ keys,
                                                          int rows_per_cta) {
    constexpr int d = 128, U = kVrU, warps = kVrThreads / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane & 7, grp = lane >> 3;
    const int r0 = blockIdx.x * rows_per_cta;
    const int r1 = min(V, r0 + rows_per_cta);
    float w[U][4][4];
    auto fetch = [&](int v0) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int v = v0 + u * 4 + grp;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (v < r1) load4_stream(W + size_t(v) * d + j * 32 + sub * 4, w[u][j]);
                else w[u][j][0] = w[u][j][1] = w[u][j][2] = w[u][j][3] = 0.f;
            }
        }
    };
    int v0 = r0 + warp * 4 * U;
    if (v0 < r1) fetch(v0);
    pdl_wait();
    pdl_trigger();
    float x[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float4 xv = *reinterpret_cast<const float4*>(xin + j * 32 + sub * 4);
        x[j][0] = xv.x; x[j][1] = xv.y; x[j][2] = xv.z; x[j][3] = xv.w;
    }
    unsigned long long best = 0ull;
    for (; v0 < r1; v0 += warps * 4 * U) {
        if (v0 != r0 + warp * 4 * U) fetch(v0);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc = fmaf(w[u][j][0], x[j][0], acc);
                acc = fmaf(w[u][j][1], x[j][1], acc);
                acc = fmaf(w[u][j][2], x[j][2], acc);
                acc = fmaf(w[u][j][3], x[j][3], acc);
            }
            const float val = group_sum(acc, 8);
            const int v = v0 + u * 4 + grp;
            if (sub == 0 && v < r1) {
                if (logits) logits[v] = val;
                best = max(best, argmax_key(val, v));
            }
        }
    }
    if (keys) {
        for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (lane == 0 && best) atomicMax(keys, best);
    }
}

// Vocab projection streamed through shared memory by the TMA engine (rows of at most 2 KiB: the dev model's
// 512-byte fp32 rows). One CTA per SM: warp kWarps (the producer) bulk-copies contiguous blocks of `rb` vocab rows
// (32 KiB) into a kVocabStages-deep ring, signalling a "full" mbarrier per stage; the kWarps consumer warps compute
// 4 rows at a time (8 lanes per row, 16-byte shared-memory reads) and release the stage on its "empty" mbarrier.
// The first blocks are requested before the PDL wait: the weights never depend on the previous kernel. All waits
// are bounded (tma.cuh): a stuck pipeline raises kErrTimeout instead of hanging.
constexpr int kVocabStages = 4;
constexpr int kVocabStageBytes = 32 * 1024;

template <typename T, int R>
__global__ void __launch_bounds__(kThreads + 32) k_vocab_tma(const float* __restrict__ xin, int nrows, int d, int V,
                                                             const T* __restrict__ W, T* __restrict__ logits,
                                                             unsigned long long* __restrict__ keys, int rb,
                                                             unsigned* err) {
    extern __shared__ __align__(128) unsigned char vsm[];
    T* stage_buf = reinterpret_cast<T*>(vsm);                                        // [kVocabStages][rb*d]
    float* xs = reinterpret_cast<float*>(vsm + size_t(kVocabStages) * kVocabStageBytes);  // [R][d]
    __shared__ uint64_t full[kVocabStages], empty[kVocabStages];
    __shared__ unsigned long long best_s[kWarps][R];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nblocks = (V + rb - 1) / rb;
    const int mine = blockIdx.x < nblocks ? (nblocks - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
    const size_t stage_elems = size_t(rb) * d;
    auto block_rows = [&](int k) { return min(rb, V - (int(blockIdx.x) + k * int(gridDim.x)) * rb); };
    auto issue = [&](int k) {
        const int s = k % kVocabStages;
        const int blk = int(blockIdx.x) + k * int(gridDim.x);
        const unsigned bytes = unsigned(block_rows(k)) * unsigned(d) * unsigned(sizeof(T));
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_load(stage_buf + s * stage_elems, W + size_t(blk) * rb * d, bytes, &full[s]);
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kVocabStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    if (warp == kWarps && lane == 0)
        for (int k = 0; k < min(kVocabStages, mine); ++k) issue(k);
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < nrows * d; i += blockDim.x) xs[i] = xin[i];
    __syncthreads();  // the last CTA-wide barrier: after it, producer and consumers never wait on each other's barriers

    if (warp == kWarps) {
        // Producer: refill each stage once all consumer warps have released it.
        if (lane == 0) {
            for (int k = kVocabStages; k < mine; ++k) {
                const int s = k % kVocabStages;
                if (!mbar_wait(&empty[s], unsigned((k / kVocabStages - 1) & 1), err)) break;
                issue(k);
            }
        }
        return;
    }
    const int sub = lane & 7, grp = lane >> 3;
    unsigned long long best[R];
#pragma unroll
    for (int r = 0; r < R; ++r) best[r] = 0ull;
    bool ok = true;
    for (int k = 0; k < mine && ok; ++k) {
        const int s = k % kVocabStages;
        ok = mbar_wait(&full[s], unsigned((k / kVocabStages) & 1), err);
        if (!ok) break;
        const T* blk = stage_buf + s * stage_elems;
        const int rows_in = block_rows(k);
        const int v_base = (int(blockIdx.x) + k * int(gridDim.x)) * rb;
        for (int r0 = warp * 4; r0 < rows_in; r0 += kWarps * 4) {
            const int row = r0 + grp;
            float acc[R];
#pragma unroll
            for (int r = 0; r < R; ++r) acc[r] = 0.f;
            if (row < rows_in) {
                for (int c = sub * 4; c < d; c += 32) {
                    float w4[4];
                    if constexpr (Store<T>::bf16) {
                        const uint2 q = *reinterpret_cast<const uint2*>(blk + size_t(row) * d + c);
                        const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
                        const float2 fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
                        w4[0] = fa.x; w4[1] = fa.y; w4[2] = fb.x; w4[3] = fb.y;
                    } else {
                        const float4 q = *reinterpret_cast<const float4*>(blk + size_t(row) * d + c);
                        w4[0] = q.x; w4[1] = q.y; w4[2] = q.z; w4[3] = q.w;
                    }
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        if (r >= nrows) break;
                        const float4 x = *reinterpret_cast<const float4*>(xs + r * d + c);
                        acc[r] = fmaf(w4[0], x.x, acc[r]);
                        acc[r] = fmaf(w4[1], x.y, acc[r]);
                        acc[r] = fmaf(w4[2], x.z, acc[r]);
                        acc[r] = fmaf(w4[3], x.w, acc[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (r >= nrows) break;
                const float val = Store<T>::round(group_sum(acc[r], 8));
                if (sub == 0 && row < rows_in) {
                    const int v = v_base + row;
                    if (logits) Store<T>::store(logits + size_t(r) * V + v, val);
                    best[r] = max(best[r], argmax_key(val, v));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (keys) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            unsigned long long b = best[r];
            for (int o = 16; o; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
            if (lane == 0) best_s[warp][r] = b;
        }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory");  // consumer warps only
    if (keys && threadIdx.x < nrows) {
        unsigned long long b = 0ull;
        for (int w = 0; w < kWarps; ++w) b = max(b, best_s[w][threadIdx.x]);
        atomicMax(keys + threadIdx.x, b);
    }
}

// ------------------------------------------------------------------------------------------------------
// Expert-grouped MoE for many tokens (d = I = 128). k_moe_up / k_moe_down give every (token, slot) its own CTAs,
// which re-run the router per CTA and re-read each expert's rows once per token; with 64+ tokens per launch that
// is ~30 MB of L2 reads per layer. Here the router runs once per token and appends (token * k + slot) to its
// expert's list; then each CTA owns a block of one expert's rows, held in registers, and walks that expert's list.
// Arithmetic, rounding points and summation orders are those of k_moe_up / k_moe_down: results are bit-identical.
constexpr int kGroupRows = 16;  // (token, slot) rows per CTA pass of a grouped kernel (the list's split over grid.z)
constexpr int kGroupTile = 4;   // rows computed together (independent reductions in flight)

// grid = ntok, block = 128. RMSNorm + gate + top-k + softmax of one token (the router of k_moe_up); the normalised
// row goes to xn_out for the grouped up-projection.
template <typename T>
__global__ void __launch_bounds__(128) k_route_rows(const float* __restrict__ x2, int ntok, Dims dm, LayerW<T> w,
                                                    float* __restrict__ xn_out, int* __restrict__ ridx,
                                                    float* __restrict__ rw, int* __restrict__ routes,
                                                    int* __restrict__ lists, int* __restrict__ counts, unsigned* err) {
    extern __shared__ float sm[];
    const int d = dm.d;
    float* xs = sm;            // [d]
    float* gl = xs + d;        // [E]
    float* misc = gl + dm.E;   // [1 + 8 + 8]: inv, indices, weights
    int* sidx = reinterpret_cast<int*>(misc + 1);
    float* sw = misc + 9;
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    for (int c = threadIdx.x; c < d; c += blockDim.x) xs[c] = x2[size_t(t) * d + c];
    __syncthreads();
    rows_rmsnorm<T>(xs, 1, d, dm.eps, w.mlp_norm, misc);
    for (int c = threadIdx.x; c < d; c += blockDim.x) xn_out[size_t(t) * d + c] = xs[c];
    for (int e0 = warp * 2; e0 < dm.E; e0 += warps * 2) {
        const T* rows[2] = {w.gate_w + size_t(e0) * d, w.gate_w + size_t(min(e0 + 1, dm.E - 1)) * d};
        const int nr = min(2, dm.E - e0);
        Frag<2> f;
        frag_load<T, 2>(f, rows, nr, d, 0);
        float acc[2][1];
        warp_gemv<T, 2, 1>(f, rows, nr, xs, d, 1, acc);
        if (lane == 0) {
            gl[e0] = Store<T>::round(__fadd_rn(acc[0][0], Store<T>::load(w.gate_b + e0)));
            if (nr > 1) gl[e0 + 1] = Store<T>::round(__fadd_rn(acc[1][0], Store<T>::load(w.gate_b + e0 + 1)));
        }
    }
    __syncthreads();
    if (warp == 0) warp_topk_softmax<T>(gl, dm.E, dm.k, sidx, sw);
    __syncthreads();
    if (threadIdx.x < dm.k) {
        const int slot = threadIdx.x;
        ridx[size_t(t) * dm.k + slot] = sidx[slot];
        rw[size_t(t) * dm.k + slot] = sw[slot];
        if (routes) routes[size_t(t) * dm.k + slot] = sidx[slot];
        const int e = int(checked_row(sidx[slot], dm.E, true, err));
        const int at = atomicAdd(counts + e, 1);
        lists[size_t(e) * ntok + at] = t * dm.k + slot;
    }
}

// The out-projection + bias + residual of k_out and the router of k_route_rows in one launch, one CTA per token, for
// programs with d = H*hd = 128 (the grouped-MoE path). Warp w owns out rows 8w .. 8w+7, each lane the same four
// elements of every row that k_out's fragments give it, so every dot product keeps k_out's order (per-lane FMA chain,
// then the warp butterfly) and the x2 row is bit-identical; then the token's norm, gate, top-k and expert-list append
// exactly as k_route_rows. Saves one dependent launch per layer.
constexpr int kOrThreads = 512;

template <typename T>
__global__ void __launch_bounds__(kOrThreads) k_out_route(const float* __restrict__ attn, const float* __restrict__ x,
                                                         int ntok, Dims dm, LayerW<T> w, float* __restrict__ x2,
                                                         float* __restrict__ xn_out, int* __restrict__ ridx,
                                                         float* __restrict__ rw, int* __restrict__ routes,
                                                         int* __restrict__ lists, int* __restrict__ counts, unsigned* err) {
    constexpr int d = 128, RPW = d / (kOrThreads / 32);
    __shared__ __align__(16) float as[d];
    __shared__ __align__(16) float xs[d];
    __shared__ float gl[kWarps * 2];
    __shared__ float misc[17];  // inv, indices, weights
    int* sidx = reinterpret_cast<int*>(misc + 1);
    float* sw = misc + 9;
    const int t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float wv[RPW][4], bv[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        load4(w.out_w + size_t(warp * RPW + i) * d + lane * 4, wv[i]);
        bv[i] = Store<T>::load(w.out_b + warp * RPW + i);
    }
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x < d) as[threadIdx.x] = attn[size_t(t) * d + threadIdx.x];
    __syncthreads();
    const float4 av = *reinterpret_cast<const float4*>(as + lane * 4);
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        float acc = 0.f;
        acc = fmaf(wv[i][0], av.x, acc);
        acc = fmaf(wv[i][1], av.y, acc);
        acc = fmaf(wv[i][2], av.z, acc);
        acc = fmaf(wv[i][3], av.w, acc);
        acc = warp_sum(acc);
        if (lane == 0) {
            const int r = warp * RPW + i;
            const size_t o = size_t(t) * d + r;
            const float v = Store<T>::round(__fadd_rn(x[o], Store<T>::round(__fadd_rn(acc, bv[i]))));
            x2[o] = v;
            xs[r] = v;
        }
    }
    __syncthreads();
    // ---- the router of k_route_rows on the x2 row
    rows_rmsnorm<T>(xs, 1, d, dm.eps, w.mlp_norm, misc);
    if (threadIdx.x < d) xn_out[size_t(t) * d + threadIdx.x] = xs[threadIdx.x];
    for (int e0 = warp * 2; e0 < dm.E; e0 += (kOrThreads / 32) * 2) {
        const T* rows[2] = {w.gate_w + size_t(e0) * d, w.gate_w + size_t(min(e0 + 1, dm.E - 1)) * d};
        const int nr = min(2, dm.E - e0);
        Frag<2> f;
        frag_load<T, 2>(f, rows, nr, d, 0);
        float acc[2][1];
        warp_gemv<T, 2, 1>(f, rows, nr, xs, d, 1, acc);
        if (lane == 0) {
            gl[e0] = Store<T>::round(__fadd_rn(acc[0][0], Store<T>::load(w.gate_b + e0)));
            if (nr > 1) gl[e0 + 1] = Store<T>::round(__fadd_rn(acc[1][0], Store<T>::load(w.gate_b + e0 + 1)));
        }
    }
    __syncthreads();
    if (warp == 0) warp_topk_softmax<T>(gl, dm.E, dm.k, sidx, sw);
    __syncthreads();
    if (threadIdx.x < dm.k) {
        const int slot = threadIdx.x;
        ridx[size_t(t) * dm.k + slot] = sidx[slot];
        rw[size_t(t) * dm.k + slot] = sw[slot];
        if (routes) routes[size_t(t) * dm.k + slot] = sidx[slot];
        const int e = int(checked_row(sidx[slot], dm.E, true, err));
        const int at = atomicAdd(counts + e, 1);
        lists[size_t(e) * ntok + at] = t * dm.k + slot;
    }
}

// grid = (E, ceil(I / kPairsPerCta), ceil(ntok / kGroupRows)), block = kThreads. Warp w holds mlp1 pairs p, p+1
// (4 rows) of expert blockIdx.x; for every (token, slot) routed there (blockIdx.z's share of the list), the SwiGLU
// of k_moe_up.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_moe_up_grouped(const float* __restrict__ xn, int ntok, Dims dm, LayerW<T> w,
                                                             const int* __restrict__ lists,
                                                             const int* __restrict__ counts, float* __restrict__ act) {
    extern __shared__ float xg[];  // [kGroupRows][d]
    __shared__ int tl[kGroupRows];  // the staged rows' (token * k + slot)
    const int e = blockIdx.x, d = dm.d;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T* W = w.w1 + size_t(e) * 2 * dm.I * d;
    const T* B = w.b1 + size_t(e) * 2 * dm.I;
    const int p = blockIdx.y * kPairsPerCta + warp * 2;
    const int np = max(0, min(2, dm.I - p));
    const int p1 = min(p + 1, dm.I - 1);
    const int p0 = min(p, dm.I - 1);
    const T* rows[4] = {W + size_t(2 * p0) * d, W + size_t(2 * p0 + 1) * d, W + size_t(2 * p1) * d,
                        W + size_t(2 * p1 + 1) * d};
    Frag<4> f;
    frag_load<T, 4>(f, rows, 2 * np, d, 0);
    float bias[4] = {0.f, 0.f, 0.f, 0.f};
    if (np > 0) {
        bias[0] = Store<T>::load(B + 2 * p0);
        bias[1] = Store<T>::load(B + 2 * p0 + 1);
        bias[2] = Store<T>::load(B + 2 * p1);
        bias[3] = Store<T>::load(B + 2 * p1 + 1);
    }
    pdl_wait();
    pdl_trigger();
    const int n = counts[e];
    for (int i0 = blockIdx.z * kGroupRows; i0 < n; i0 += gridDim.z * kGroupRows) {
        const int rows_here = min(kGroupRows, n - i0);
        __syncthreads();
        for (int r = threadIdx.x; r < rows_here; r += blockDim.x) tl[r] = lists[size_t(e) * ntok + i0 + r];
        __syncthreads();
        for (int i = threadIdx.x; i < rows_here * (d / 4); i += blockDim.x) {
            const int r = i / (d / 4), c = (i % (d / 4)) * 4;
            const int tok = tl[r] / dm.k;
            *reinterpret_cast<float4*>(xg + r * d + c) = *reinterpret_cast<const float4*>(xn + size_t(tok) * d + c);
        }
        __syncthreads();
        if (np == 0) continue;
        for (int r0 = 0; r0 < rows_here; r0 += kGroupTile) {
            const int tt = min(kGroupTile, rows_here - r0);
            float acc[4][kGroupTile];
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int t = 0; t < kGroupTile; ++t) acc[u][t] = 0.f;
            frag_fma<4, kGroupTile>(f, xg + r0 * d, d, tt, 0, acc);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int t = 0; t < kGroupTile; ++t) acc[u][t] = warp_sum(acc[u][t]);
            // Lane q < 2 * tt handles row r0 + q / 2, pair p + q % 2.
            const int q = lane;
            if (q < 2 * tt && q % 2 < np) {
                const int t = q / 2, h = q % 2;
                float ag = 0.f, al = 0.f;
#pragma unroll
                for (int tq = 0; tq < kGroupTile; ++tq)
                    if (tq == t) {
                        ag = h == 0 ? acc[0][tq] : acc[2][tq];
                        al = h == 0 ? acc[1][tq] : acc[3][tq];
                    }
                const float bg = h == 0 ? bias[0] : bias[2];
                const float bl = h == 0 ? bias[1] : bias[3];
                const float hg = Store<T>::round(__fadd_rn(Store<T>::round(ag), bg));
                const float hl = Store<T>::round(__fadd_rn(Store<T>::round(al), bl));
                const float glu = fminf(hg, dm.limit);
                const float lin = fminf(fmaxf(hl, -dm.limit), dm.limit);
                const float z = Store<T>::round(__fmul_rn(glu, dm.alpha));
                const float sg = Store<T>::round(1.0f / (1.0f + expf(-z)));
                const float og = Store<T>::round(__fmul_rn(glu, sg));
                const float l1 = Store<T>::round(__fadd_rn(lin, 1.0f));
                act[size_t(tl[r0 + t]) * dm.I + p + h] = Store<T>::round(__fmul_rn(og, l1));
            }
        }
    }
}

// grid = (E, ceil(d / kWarps), ceil(ntok / kGroupRows)), block = kThreads. Warp w holds mlp2 row (e, c) of expert
// blockIdx.x; for every (token, slot) routed there (blockIdx.z's share), y = mlp2 . act + bias (the per-slot term of
// k_moe_down) into ys.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_moe_down_grouped(const float* __restrict__ act, int ntok, Dims dm,
                                                               const T* __restrict__ w2, const T* __restrict__ b2,
                                                               const int* __restrict__ lists,
                                                               const int* __restrict__ counts, float* __restrict__ ys) {
    extern __shared__ float ag[];  // [kGroupRows][I]
    __shared__ int tl[kGroupRows];  // the staged rows' (token * k + slot)
    const int e = blockIdx.x, I = dm.I;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.y * kWarps + warp;
    const int cc = min(c, dm.d - 1);
    const T* rows[1] = {w2 + (size_t(e) * dm.d + cc) * I};
    Frag<1> f;
    frag_load<T, 1>(f, rows, c < dm.d ? 1 : 0, I, 0);
    const float bias = Store<T>::load(b2 + size_t(e) * dm.d + cc);
    pdl_wait();
    pdl_trigger();
    const int n = counts[e];
    for (int i0 = blockIdx.z * kGroupRows; i0 < n; i0 += gridDim.z * kGroupRows) {
        const int rows_here = min(kGroupRows, n - i0);
        __syncthreads();
        for (int r = threadIdx.x; r < rows_here; r += blockDim.x) tl[r] = lists[size_t(e) * ntok + i0 + r];
        __syncthreads();
        for (int i = threadIdx.x; i < rows_here * (I / 4); i += blockDim.x) {
            const int r = i / (I / 4), q = (i % (I / 4)) * 4;
            *reinterpret_cast<float4*>(ag + r * I + q) = *reinterpret_cast<const float4*>(act + size_t(tl[r]) * I + q);
        }
        __syncthreads();
        if (c >= dm.d) continue;
        for (int r0 = 0; r0 < rows_here; r0 += kGroupTile) {
            const int tt = min(kGroupTile, rows_here - r0);
            float acc[1][kGroupTile];
#pragma unroll
            for (int t = 0; t < kGroupTile; ++t) acc[0][t] = 0.f;
            frag_fma<1, kGroupTile>(f, ag + r0 * I, I, tt, 0, acc);
#pragma unroll
            for (int t = 0; t < kGroupTile; ++t) acc[0][t] = warp_sum(acc[0][t]);
            if (lane < tt) {
                float part = acc[0][0];
#pragma unroll
                for (int t = 1; t < kGroupTile; ++t)
                    if (t == lane) part = acc[0][t];
                ys[size_t(tl[r0 + lane]) * dm.d + c] = Store<T>::round(__fadd_rn(Store<T>::round(part), bias));
            }
        }
    }
}

// grid = ntok, block = d (<= 1024). x = x2 + the routing-weighted sum of the slots' ys in slot order (the combine of
// k_moe_down); CTA 0 also clears the per-expert counts for the next layer's router.
template <typename T>
__global__ void k_moe_combine_rows(const float* __restrict__ ys, const float* __restrict__ x2, int ntok, Dims dm,
                                   const float* __restrict__ rw, float* __restrict__ x_out, int* __restrict__ counts) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x, c = threadIdx.x;
    if (t == 0 && c < dm.E) counts[c] = 0;
    if (c >= dm.d) return;
    float comb = 0.f;
    for (int u = 0; u < dm.k; ++u)
        comb = __fadd_rn(comb, __fmul_rn(ys[(size_t(t) * dm.k + u) * dm.d + c], rw[size_t(t) * dm.k + u]));
    x_out[size_t(t) * dm.d + c] = Store<T>::round(__fadd_rn(x2[size_t(t) * dm.d + c], Store<T>::round(comb)));
}

// Vocab projection of many rows (fp32, d = 128): one pass over the vocab matrix for up to kVtRows activation rows.
// Each CTA keeps the rows in shared memory and walks 128-row vocab tiles (cp.async double buffer, 132-float padded
// rows: conflict-free 16-byte reads); thread (ty, tx) computes kVtRows/16 rows x 8 vocab rows (tx + 16j), each dot
// product one sequential FMA chain over the 128 features. The greedy argmax is kept per thread across tiles and
// merged with one 64-bit atomicMax per (CTA, row). Compute-bound: 2 * rows * V * 128 FLOP, weights read once.
constexpr int kVtRows = 64;
constexpr int kVtVocab = 128;
constexpr int kVtD = 128;
constexpr int kVtPad = kVtD + 4;
constexpr size_t kVtSmemBytes = (size_t(kVtRows) + 2 * kVtVocab) * kVtPad * 4;

__global__ void __launch_bounds__(kThreads, 1) k_vocab_tiled(const float* __restrict__ xin, int nrows, int V,
                                                             const float* __restrict__ W, float* __restrict__ logits,
                                                             unsigned long long* __restrict__ keys) {
    extern __shared__ __align__(16) float vt[];
    float* xs = vt;                          // [kVtRows][kVtPad]
    float* ws = vt + kVtRows * kVtPad;       // [2][kVtVocab][kVtPad]
    constexpr int RPT = kVtRows / 16;        // rows per thread
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int tiles = (V + kVtVocab - 1) / kVtVocab;
    auto load_tile = [&](int tile, int buf) {
        float* dst = ws + buf * kVtVocab * kVtPad;
        for (int i = threadIdx.x; i < kVtVocab * (kVtD / 4); i += blockDim.x) {
            const int r = i / (kVtD / 4), c = (i % (kVtD / 4)) * 4;
            const int v = tile * kVtVocab + r;
            if (v < V) cp_async16(dst + r * kVtPad + c, W + size_t(v) * kVtD + c);
        }
        cp_async_commit();
    };
    int tile = blockIdx.x;
    if (tile < tiles) load_tile(tile, 0);  // weights: before the PDL wait
    pdl_wait();
    pdl_trigger();
    for (int r0 = 0; r0 < nrows; r0 += kVtRows) {
        const int rr = min(kVtRows, nrows - r0);
        __syncthreads();
        for (int i = threadIdx.x; i < kVtRows * (kVtD / 4); i += blockDim.x) {
            const int r = i / (kVtD / 4), c = (i % (kVtD / 4)) * 4;
            const float4 v = r < rr ? *reinterpret_cast<const float4*>(xin + size_t(r0 + r) * kVtD + c)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(xs + r * kVtPad + c) = v;
        }
        unsigned long long best[RPT];
#pragma unroll
        for (int i = 0; i < RPT; ++i) best[i] = 0ull;
        if (r0 > 0) {
            tile = blockIdx.x;
            if (tile < tiles) load_tile(tile, 0);
        }
        for (int it = 0; tile < tiles; ++it, tile += gridDim.x) {
            const int buf = it & 1;
            const int next = tile + gridDim.x;
            if (next < tiles) {
                load_tile(next, buf ^ 1);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncthreads();
            const float* wt = ws + buf * kVtVocab * kVtPad;
            float acc[RPT][8];
#pragma unroll
            for (int i = 0; i < RPT; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
#pragma unroll 4
            for (int k = 0; k < kVtD; k += 4) {
                float4 x[RPT], w[8];
#pragma unroll
                for (int i = 0; i < RPT; ++i) x[i] = *reinterpret_cast<const float4*>(xs + (ty * RPT + i) * kVtPad + k);
#pragma unroll
                for (int j = 0; j < 8; ++j) w[j] = *reinterpret_cast<const float4*>(wt + (tx + 16 * j) * kVtPad + k);
#pragma unroll
                for (int i = 0; i < RPT; ++i)
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        acc[i][j] = fmaf(x[i].x, w[j].x, acc[i][j]);
                        acc[i][j] = fmaf(x[i].y, w[j].y, acc[i][j]);
                        acc[i][j] = fmaf(x[i].z, w[j].z, acc[i][j]);
                        acc[i][j] = fmaf(x[i].w, w[j].w, acc[i][j]);
                    }
            }
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                const int row = ty * RPT + i;
                if (row >= rr) continue;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int v = tile * kVtVocab + tx + 16 * j;
                    if (v < V) {
                        if (logits) logits[size_t(r0 + row) * V + v] = acc[i][j];
                        best[i] = max(best[i], argmax_key(acc[i][j], v));
                    }
                }
            }
            __syncthreads();  // the buffer is refilled two tiles later
        }
        if (keys) {
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                unsigned long long b = best[i];
#pragma unroll
                for (int o = 8; o; o >>= 1) b = max(b, __shfl_xor_sync(0xffffffffu, b, o));
                const int row = ty * RPT + i;
                if (tx == 0 && row < rr && b) atomicMax(keys + r0 + row, b);
            }
        }
    }
}

}  // namespace cb200
