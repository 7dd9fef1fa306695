// Flash attention for prefill chunks (head_dim 64, bf16), the reference's sink attention
// (chroma/models/gpt_oss.py:133-151, chroma/models/cached.py:36-47) without materialising the score matrix:
//
//   out[i] = sum_j softmax_j([s_i0 .. s_ij .., sink]) v_j,  s_ij = q_i . k_j / sqrt(64) (masked to -inf)
//
// One CTA = 128 query rows of one head of one sequence, 8 warps x 16 rows. Keys come in 64-row tiles, first the ring
// cache (visible when its slot's position is <= the query's and inside the window; tiles with no live slot are
// never loaded) then the chunk's own rows (causal, windowed). S = Q K^T and O += P V run on mma.sync m16n8k16 (bf16 in,
// fp32 accumulate); the online softmax keeps a running max and sum per row; the sink logit joins the final
// normalisation. K/V tiles are double-buffered with cp.async into XOR-swizzled shared memory read by ldmatrix.
#pragma once

#include "tma.cuh"

namespace cb200 {

constexpr int kFaRows = 128;  // query rows per CTA (8 warps x 16)
constexpr int kFaKeys = 64;  // keys per tile
constexpr int kFaDim = 64;   // head_dim

struct FlashArgs {
    int n, ctx, B, H, KV, G;
    size_t cache_seq_stride;  // elements between sequences in the cache (layer offset applied)
    int window;               // 0 = none
    float scale_log2;         // sm_scale * log2(e)
    const int64_t* slots;     // [B][ctx] ring-slot positions (-1 empty), or nullptr when ctx == 0
    const int64_t* pos0;      // [B] position of each sequence's first new row (nullptr: 0)
};

__device__ __forceinline__ uint32_t fa_swz(int row, int col) {  // element offset in a [64][64] bf16 tile
    return uint32_t(row * 64 + (((col >> 3) ^ (row & 7)) << 3) + (col & 7));
}


__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 2^x on the special-function unit (ex2.approx, flush-to-zero): 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Shared memory of one CTA (dynamic): Q tile, double-buffered K and V tiles, key positions, the list of live cache
// tiles and its bitmask.
constexpr int kFaThreads = 32 * (kFaRows / 16);
constexpr int kFaMaxCacheTiles = 1024;  // ring contexts up to 65,536 positions
constexpr size_t kFaSmemBytes = size_t(kFaRows) * kFaDim * 2 + 4 * size_t(kFaKeys) * kFaDim * 2 +
                                2 * kFaKeys * sizeof(int64_t) + kFaMaxCacheTiles * sizeof(uint16_t) +
                                (kFaMaxCacheTiles / 32) * sizeof(uint32_t);

// grid = (ceil(n / kFaRows), H, B); block = kFaThreads; dynamic shared memory kFaSmemBytes.
//
// Only tiles holding a key some row of the block can see are loaded: cache tiles are screened against the ring-slot
// positions first (a fresh sequence has none), and the chunk's own tiles start at the window's edge. Tiles whose
// every key is visible to every row (below the diagonal, inside the window) skip the per-element mask.
__global__ void __launch_bounds__(kFaThreads, 2) k_flash_prefill(const __nv_bfloat16* __restrict__ q, FlashArgs a,
                                                                 const __nv_bfloat16* __restrict__ cache_k,
                                                                 const __nv_bfloat16* __restrict__ cache_v,
                                                                 const __nv_bfloat16* __restrict__ new_k,
                                                                 const __nv_bfloat16* __restrict__ new_v,
                                                                 const __nv_bfloat16* __restrict__ sinks,
                                                                 __nv_bfloat16* __restrict__ out) {
    extern __shared__ __align__(128) uint8_t fa_smem[];
    __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(fa_smem);
    __nv_bfloat16* Ks0 = Qs + kFaRows * kFaDim;
    __nv_bfloat16* Vs0 = Ks0 + 2 * kFaKeys * kFaDim;
    int64_t* tslot0 = reinterpret_cast<int64_t*>(Vs0 + 2 * kFaKeys * kFaDim);
    uint16_t* live_list = reinterpret_cast<uint16_t*>(tslot0 + 2 * kFaKeys);
    uint32_t* live_bits = reinterpret_cast<uint32_t*>(live_list + kFaMaxCacheTiles);
    __shared__ int s_nlive;

    const int qb = gridDim.x - 1 - blockIdx.x;  // heavy (late) query blocks first
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / a.G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int i0 = qb * kFaRows;
    const int i_last = min(i0 + kFaRows, a.n) - 1;  // last real query row of the block
    const size_t row_stride = size_t(a.KV) * kFaDim;  // elements between consecutive key rows
    const __nv_bfloat16* ck = cache_k + b * a.cache_seq_stride + size_t(kvh) * kFaDim;
    const __nv_bfloat16* cv = cache_v + b * a.cache_seq_stride + size_t(kvh) * kFaDim;
    const __nv_bfloat16* nk = new_k + (size_t(b) * a.n * a.KV + kvh) * kFaDim;
    const __nv_bfloat16* nv = new_v + (size_t(b) * a.n * a.KV + kvh) * kFaDim;

    const int cache_tiles = (a.ctx + kFaKeys - 1) / kFaKeys;
    for (int w = threadIdx.x; w < (cache_tiles + 31) / 32; w += blockDim.x) live_bits[w] = 0;
    pdl_wait();
    pdl_trigger();
    const int64_t p0 = a.pos0 ? a.pos0[b] : 0;
    const int64_t first = p0 + i0, last = p0 + i_last;
    // Q tile -> shared memory (rows past n are zero).
    for (int e = threadIdx.x; e < kFaRows * 8; e += blockDim.x) {
        const int r = e >> 3, c = (e & 7) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (i0 + r < a.n) v = *reinterpret_cast<const uint4*>(q + ((size_t(b) * a.n + i0 + r) * a.H + h) * kFaDim + c);
        *reinterpret_cast<uint4*>(Qs + fa_swz(r, c)) = v;
    }
    // Screen the ring: a cache tile is live when one of its slots holds a position some row of the block can see.
    __syncthreads();
    for (int j = threadIdx.x; j < a.ctx; j += blockDim.x) {
        const int64_t tj = a.slots[size_t(b) * a.ctx + j];
        if (tj >= 0 && tj <= last && (a.window <= 0 || tj > first - a.window))
            atomicOr(&live_bits[(j / kFaKeys) >> 5], 1u << ((j / kFaKeys) & 31));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int nl = 0;
        for (int w = 0; w < (cache_tiles + 31) / 32; ++w) {
            uint32_t bits = live_bits[w];
            while (bits) {
                const int bit = __ffs(bits) - 1;
                bits &= bits - 1;
                live_list[nl++] = uint16_t(w * 32 + bit);
            }
        }
        s_nlive = nl;
    }
    __syncthreads();
    const int nlive = s_nlive;
    // The chunk's own tiles: from the window's edge (row i sees own key j iff j <= i and j > i - window) to the
    // tile holding the block's last row.
    const int own_lo = a.window > 0 ? max(0, i0 - a.window + 1) / kFaKeys : 0;
    const int own_hi = (i_last + kFaKeys) / kFaKeys;
    const int tiles = nlive + max(0, own_hi - own_lo);

    // Tile index -> (cached?, first key row).
    auto tile_key0 = [&](int tile, bool& cached) {
        cached = tile < nlive;
        return (cached ? int(live_list[tile]) : own_lo + tile - nlive) * kFaKeys;
    };
    auto load_tile = [&](int tile, int buf) {
        bool cached;
        const int j0 = tile_key0(tile, cached);
        const int limit = cached ? a.ctx : a.n;
        const __nv_bfloat16* kb = cached ? ck : nk;
        const __nv_bfloat16* vb = cached ? cv : nv;
        __nv_bfloat16* Kd = Ks0 + buf * kFaKeys * kFaDim;
        __nv_bfloat16* Vd = Vs0 + buf * kFaKeys * kFaDim;
        for (int e = threadIdx.x; e < kFaKeys * 8; e += blockDim.x) {
            const int r = e >> 3, c = (e & 7) * 8;
            if (j0 + r < limit) {
                cp_async16(Kd + fa_swz(r, c), kb + size_t(j0 + r) * row_stride + c);
                cp_async16(Vd + fa_swz(r, c), vb + size_t(j0 + r) * row_stride + c);
            } else {
                *reinterpret_cast<uint4*>(Kd + fa_swz(r, c)) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(Vd + fa_swz(r, c)) = make_uint4(0, 0, 0, 0);
            }
        }
        if (threadIdx.x < kFaKeys) {
            const int j = j0 + threadIdx.x;
            // Absolute position of each key (-1: not a key).
            tslot0[buf * kFaKeys + threadIdx.x] = j < limit ? (cached ? a.slots[size_t(b) * a.ctx + j] : p0 + j) : -1;
        }
        cp_async_commit();
    };
    if (tiles > 0) load_tile(0, 0);

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    const int r_lo = warp * 16 + g;  // this thread's two query rows within the block: r_lo, r_lo + 8
    const int64_t t_lo = p0 + i0 + r_lo;  // position of row r_lo (row r_lo + 8: t_lo + 8)
    const bool row_ok[2] = {i0 + r_lo < a.n, i0 + r_lo + 8 < a.n};
    uint32_t qf[4][4];

    for (int tile = 0; tile < tiles; ++tile) {
        const int buf = tile & 1;
        if (tile + 1 < tiles) {
            load_tile(tile + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (tile == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int col = kk * 16 + 8 * (lane >> 4);
                ldsm_x4(qf[kk], Qs + fa_swz(row, col));
            }
        }
        const __nv_bfloat16* Kb = Ks0 + buf * kFaKeys * kFaDim;
        const __nv_bfloat16* Vb = Vs0 + buf * kFaKeys * kFaDim;
        const int64_t* ts = tslot0 + buf * kFaKeys;
        bool cached;
        const int j0 = tile_key0(tile, cached);
        // Every key of an own tile is visible to every row when the tile ends at or before the first row and starts
        // inside the last row's window.
        const bool masked = cached || j0 + kFaKeys - 1 > i0 || (a.window > 0 && j0 <= i_last - a.window);

        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int nt = 0; nt < 8; nt += 2) {
                uint32_t kf[4];
                const int key = nt * 8 + (lane & 7) + 8 * (lane >> 4);
                const int col = kk * 16 + 8 * ((lane >> 3) & 1);
                ldsm_x4(kf, Kb + fa_swz(key, col));
                mma_bf16(s[nt], qf[kk], kf[0], kf[1]);
                mma_bf16(s[nt + 1], qf[kk], kf[2], kf[3]);
            }
        }
        // Mask, then the online softmax in the log2 domain: the running max m_run is kept scaled, so each
        // probability is one FMA and one ex2: p = 2^(s * scale - m).
        float mx[2] = {-INFINITY, -INFINITY};
        if (masked) {
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int rr = e >> 1;  // 0: row r_lo, 1: row r_lo + 8
                    const int64_t tj = ts[nt * 8 + 2 * t4 + (e & 1)];
                    const int64_t t_i = t_lo + 8 * rr;
                    const bool vis = tj >= 0 && tj <= t_i && (a.window <= 0 || tj > t_i - a.window) && row_ok[rr];
                    s[nt][e] = vis ? s[nt][e] : -INFINITY;
                    mx[rr] = fmaxf(mx[rr], s[nt][e]);
                }
            }
        } else {
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                mx[0] = fmaxf(mx[0], fmaxf(s[nt][0], s[nt][1]));
                mx[1] = fmaxf(mx[1], fmaxf(s[nt][2], s[nt][3]));
            }
        }
        float corr[2], neg[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
            const float m_new = fmaxf(m_run[rr], mx[rr] * a.scale_log2);
            const bool none = m_new == -INFINITY;  // no visible key for this row yet
            corr[rr] = none ? 1.f : fast_exp2(m_run[rr] - m_new);
            neg[rr] = none ? 0.f : -m_new;
            m_run[rr] = m_new;
        }
        uint32_t pf[4][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                p[e] = fast_exp2(fmaf(s[nt][e], a.scale_log2, neg[e >> 1]));
                rs[e >> 1] += p[e];
            }
            const int ks = nt >> 1, hi = nt & 1;
            pf[ks][hi * 2 + 0] = pack_bf16(p[0], p[1]);
            pf[ks][hi * 2 + 1] = pack_bf16(p[2], p[3]);
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) l_run[rr] = l_run[rr] * corr[rr] + rs[rr];
        if (__any_sync(0xffffffffu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
            for (int nd = 0; nd < 8; ++nd) {
                o[nd][0] *= corr[0];
                o[nd][1] *= corr[0];
                o[nd][2] *= corr[1];
                o[nd][3] *= corr[1];
            }
        }
        // A-fragment order of P for k-step ks: {rows g / keys 2t, rows g+8 / keys 2t, rows g / keys 2t+8, ...}.
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const uint32_t af[4] = {pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3]};
#pragma unroll
            for (int nd = 0; nd < 8; nd += 2) {
                uint32_t vf[4];
                const int key = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int col = nd * 8 + 8 * (lane >> 4);
                ldsm_x4_t(vf, Vb + fa_swz(key, col));
                mma_bf16(o[nd], af, vf[0], vf[1]);
                mma_bf16(o[nd + 1], af, vf[2], vf[3]);
            }
        }
        __syncthreads();
    }
    // Row sums across the quad, the sink logit, normalise and store.
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 1);
        l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 2);
    }
    const float sink = __bfloat162float(sinks[h]) * 1.4426950408889634f;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int i = i0 + r_lo + 8 * rr;
        if (i >= a.n) continue;
        const float mf = fmaxf(m_run[rr], sink);
        const float c = m_run[rr] == -INFINITY ? 0.f : exp2f(m_run[rr] - mf);
        const float inv = 1.0f / (l_run[rr] * c + exp2f(sink - mf));
        __nv_bfloat16* orow = out + ((size_t(b) * a.n + i) * a.H + h) * kFaDim;
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
            const float v0 = o[nd][2 * rr] * c * inv, v1 = o[nd][2 * rr + 1] * c * inv;
            *reinterpret_cast<__nv_bfloat162*>(orow + nd * 8 + 2 * t4) = __floats2bfloat162_rn(v0, v1);
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Flash decoding: attention of a few new rows per sequence (n * G <= 16 query rows, one KV head's query group)
// against the ring cache, split over the keys.
//
// grid = (B, KV, splits); block = 4 warps. The M = 16 rows of the tensor-core tile are the n x G query rows that
// share one KV head (GQA packs them, so each K/V byte read from HBM feeds G heads). The CTA streams 64-key tiles of
// its key range through a 3-stage cp.async ring; warp w takes keys [16w, 16w + 16) of every tile and keeps its own
// online softmax. At the end the 4 warps merge in shared memory; the split's (max, sum, output) rows go to `part`,
// and the last split CTA of (sequence, KV head) to finish merges all splits with the sink logit and writes the
// output (splits == 1: directly). The chunk's own new rows join the last split as one extra tile.
constexpr int kFdRows = 16;
constexpr int kFdKeys = 64;
constexpr int kFdStages = 3;
constexpr int kFdThreads = 128;
constexpr size_t kFdSmemBytes = size_t(kFdRows) * kFaDim * 2 +
                                size_t(kFdStages) * (2 * kFdKeys * kFaDim * 2 + kFdKeys * sizeof(int64_t));

struct DecodeArgs {
    int n, ctx, B, H, KV, G, splits, split_keys;  // split_keys: cache keys per split (a multiple of 64)
    size_t cache_seq_stride;
    int window;
    float scale_log2;
    const int64_t* slots;   // [B][ctx] ring-slot positions (-1 empty)
    const int64_t* pos0;    // [B] position of each sequence's first new row
    float* part;            // [B][KV][splits][16][2 + 64]
    unsigned* counters;     // [B][KV], zero between launches
};

__global__ void __launch_bounds__(kFdThreads) k_flash_decode(const __nv_bfloat16* __restrict__ q, DecodeArgs a,
                                                             const __nv_bfloat16* __restrict__ cache_k,
                                                             const __nv_bfloat16* __restrict__ cache_v,
                                                             const __nv_bfloat16* __restrict__ new_k,
                                                             const __nv_bfloat16* __restrict__ new_v,
                                                             const __nv_bfloat16* __restrict__ sinks,
                                                             __nv_bfloat16* __restrict__ out) {
    extern __shared__ __align__(128) uint8_t fd_smem[];
    __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(fd_smem);
    __nv_bfloat16* Ks0 = Qs + kFdRows * kFaDim;
    __nv_bfloat16* Vs0 = Ks0 + kFdStages * kFdKeys * kFaDim;
    int64_t* ts0 = reinterpret_cast<int64_t*>(Vs0 + kFdStages * kFdKeys * kFaDim);
    __shared__ bool s_last;

    const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int rows = a.n * a.G;  // real query rows (<= 16)
    const size_t row_stride = size_t(a.KV) * kFaDim;
    const __nv_bfloat16* ck = cache_k + b * a.cache_seq_stride + size_t(kvh) * kFaDim;
    const __nv_bfloat16* cv = cache_v + b * a.cache_seq_stride + size_t(kvh) * kFaDim;
    const __nv_bfloat16* nk = new_k + (size_t(b) * a.n * a.KV + kvh) * kFaDim;
    const __nv_bfloat16* nv = new_v + (size_t(b) * a.n * a.KV + kvh) * kFaDim;

    pdl_wait();
    pdl_trigger();
    const int64_t p0 = a.pos0[b];
    // Q rows: row r = i * G + gh is query row i of head kvh * G + gh (rows >= n * G are zero).
    for (int e = threadIdx.x; e < kFdRows * 8; e += blockDim.x) {
        const int r = e >> 3, c = (e & 7) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < rows) {
            const int i = r / a.G, h = kvh * a.G + r % a.G;
            v = *reinterpret_cast<const uint4*>(q + ((size_t(b) * a.n + i) * a.H + h) * kFaDim + c);
        }
        *reinterpret_cast<uint4*>(Qs + fa_swz(r, c)) = v;
    }
    const int j_begin = split * a.split_keys, j_end = min(a.ctx, j_begin + a.split_keys);
    const int cache_tiles = j_end > j_begin ? (j_end - j_begin + kFdKeys - 1) / kFdKeys : 0;
    const bool own = split == a.splits - 1;
    const int tiles = cache_tiles + (own ? 1 : 0);  // n <= 16 < 64: the own rows fit one tile

    auto load_tile = [&](int tile, int stage) {
        const bool cached = tile < cache_tiles;
        const int j0 = cached ? j_begin + tile * kFdKeys : 0;
        const int limit = cached ? j_end : a.n;
        const __nv_bfloat16* kb = cached ? ck : nk;
        const __nv_bfloat16* vb = cached ? cv : nv;
        __nv_bfloat16* Kd = Ks0 + stage * kFdKeys * kFaDim;
        __nv_bfloat16* Vd = Vs0 + stage * kFdKeys * kFaDim;
        for (int e = threadIdx.x; e < kFdKeys * 8; e += blockDim.x) {
            const int r = e >> 3, c = (e & 7) * 8;
            if (j0 + r < limit) {
                cp_async16(Kd + fa_swz(r, c), kb + size_t(j0 + r) * row_stride + c);
                cp_async16(Vd + fa_swz(r, c), vb + size_t(j0 + r) * row_stride + c);
            } else {
                *reinterpret_cast<uint4*>(Kd + fa_swz(r, c)) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(Vd + fa_swz(r, c)) = make_uint4(0, 0, 0, 0);
            }
        }
        if (threadIdx.x < kFdKeys) {
            const int j = j0 + threadIdx.x;
            ts0[stage * kFdKeys + threadIdx.x] = j < limit ? (cached ? a.slots[size_t(b) * a.ctx + j] : p0 + j) : -1;
        }
    };
    // Prologue: stages 0 .. kFdStages-2 in flight (one commit group per stage, empty groups keep the count).
#pragma unroll
    for (int st = 0; st < kFdStages - 1; ++st) {
        if (st < tiles) load_tile(st, st);
        cp_async_commit();
    }

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    // This thread's rows g and g + 8: their positions (-1 marks a padding row).
    int64_t t_row[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int r = g + 8 * rr;
        t_row[rr] = r < rows ? p0 + r / a.G : -1;
    }
    uint32_t qf[4][4];

    for (int tile = 0; tile < tiles; ++tile) {
        const int stage = tile % kFdStages;
        {
            const int ahead = tile + kFdStages - 1;
            if (ahead < tiles) load_tile(ahead, ahead % kFdStages);
            cp_async_commit();
        }
        cp_async_wait<kFdStages - 1>();
        __syncthreads();
        if (tile == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
                const int col = kk * 16 + 8 * (lane >> 4);
                ldsm_x4(qf[kk], Qs + fa_swz(row, col));
            }
        }
        const __nv_bfloat16* Kb = Ks0 + stage * kFdKeys * kFaDim;
        const __nv_bfloat16* Vb = Vs0 + stage * kFdKeys * kFaDim;
        const int64_t* ts = ts0 + stage * kFdKeys;
        const int kw = warp * 16;  // this warp's 16 keys of the tile

        float sc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t kf[4];
            const int key = kw + (lane & 7) + 8 * (lane >> 4);
            const int col = kk * 16 + 8 * ((lane >> 3) & 1);
            ldsm_x4(kf, Kb + fa_swz(key, col));
            mma_bf16(sc[0], qf[kk], kf[0], kf[1]);
            mma_bf16(sc[1], qf[kk], kf[2], kf[3]);
        }
        float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int rr = e >> 1;
                const int64_t tj = ts[kw + nt * 8 + 2 * t4 + (e & 1)];
                const int64_t ti = t_row[rr];
                const bool vis = ti >= 0 && tj >= 0 && tj <= ti && (a.window <= 0 || tj > ti - a.window);
                // The reference stores q.k in bf16 before scaling (gpt_oss.py:133-151 in a bf16 graph).
                sc[nt][e] = vis ? bf16_round(sc[nt][e]) : -INFINITY;
                mx[rr] = fmaxf(mx[rr], sc[nt][e]);
            }
        }
        float corr[2], neg[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
            mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
            const float m_new = fmaxf(m_run[rr], mx[rr] * a.scale_log2);
            const bool none = m_new == -INFINITY;
            corr[rr] = none ? 1.f : fast_exp2(m_run[rr] - m_new);
            neg[rr] = none ? 0.f : -m_new;
            m_run[rr] = m_new;
        }
        uint32_t af[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                pv[e] = fast_exp2(fmaf(sc[nt][e], a.scale_log2, neg[e >> 1]));
                rs[e >> 1] += pv[e];
            }
            af[nt * 2 + 0] = pack_bf16(pv[0], pv[1]);
            af[nt * 2 + 1] = pack_bf16(pv[2], pv[3]);
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) l_run[rr] = l_run[rr] * corr[rr] + rs[rr];
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
            o[nd][0] *= corr[0];
            o[nd][1] *= corr[0];
            o[nd][2] *= corr[1];
            o[nd][3] *= corr[1];
        }
#pragma unroll
        for (int nd = 0; nd < 8; nd += 2) {
            uint32_t vf[4];
            const int key = kw + (lane & 7) + 8 * ((lane >> 3) & 1);
            const int col = nd * 8 + 8 * (lane >> 4);
            ldsm_x4_t(vf, Vb + fa_swz(key, col));
            mma_bf16(o[nd], af, vf[0], vf[1]);
            mma_bf16(o[nd + 1], af, vf[2], vf[3]);
        }
        __syncthreads();  // the stage is refilled kFdStages - 1 tiles later
    }
    cp_async_wait<0>();
    __syncthreads();

    // Merge the 4 warps (shared memory reused: [warp][16 rows][64] outputs, then max and sum per warp and row).
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 1);
        l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 2);
    }
    float* wo = reinterpret_cast<float*>(Ks0);              // 4 x 16 x 64 floats = 16 KB
    float* wm = wo + 4 * kFdRows * kFaDim;                   // 4 x 16
    float* wl = wm + 4 * kFdRows;                            // 4 x 16
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = g + 8 * (e >> 1), c = nd * 8 + 2 * t4 + (e & 1);
            wo[(warp * kFdRows + r) * kFaDim + c] = o[nd][e];
        }
    }
    if (t4 == 0) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            wm[warp * kFdRows + g + 8 * rr] = m_run[rr];
            wl[warp * kFdRows + g + 8 * rr] = l_run[rr];
        }
    }
    __syncthreads();
    float* pp = a.part + ((size_t(b) * a.KV + kvh) * a.splits + split) * kFdRows * (2 + kFaDim);
    // Thread -> (row, 8 columns): 16 rows x 8 column groups = 128 threads.
    {
        const int r = threadIdx.x >> 3, c0 = (threadIdx.x & 7) * 8;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w * kFdRows + r]);
        float L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float mw = wm[w * kFdRows + r];
            const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
            L += wl[w * kFdRows + r] * f;
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] += wo[(w * kFdRows + r) * kFaDim + c0 + c] * f;
        }
        if (c0 == 0) {
            pp[r * (2 + kFaDim) + 0] = M;
            pp[r * (2 + kFaDim) + 1] = L;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) pp[r * (2 + kFaDim) + 2 + c0 + c] = acc[c];
    }
    // Last split CTA of this (sequence, KV head) merges the splits with the sink.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* counter = a.counters + size_t(b) * a.KV + kvh;
        const unsigned prev = atomicAdd(counter, 1u);
        s_last = prev == unsigned(a.splits - 1);
        if (s_last) *counter = 0u;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = a.part + (size_t(b) * a.KV + kvh) * a.splits * kFdRows * (2 + kFaDim);
    const int r = threadIdx.x >> 3, c0 = (threadIdx.x & 7) * 8;
    if (r >= rows) return;
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, __ldcg(base + (size_t(sp) * kFdRows + r) * (2 + kFaDim)));
    const int h = kvh * a.G + r % a.G, i = r / a.G;
    const float sink = __bfloat162float(sinks[h]) * 1.4426950408889634f;
    const float mf = fmaxf(M, sink);
    float L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < a.splits; ++sp) {
        const float* row = base + (size_t(sp) * kFdRows + r) * (2 + kFaDim);
        const float ms = __ldcg(row);
        const float f = ms == -INFINITY ? 0.f : exp2f(ms - mf);
        L += __ldcg(row + 1) * f;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] += __ldcg(row + 2 + c0 + c) * f;
    }
    const float inv = 1.0f / (L + exp2f(sink - mf));
    __nv_bfloat16* orow = out + ((size_t(b) * a.n + i) * a.H + h) * kFaDim + c0;
    uint4 packed;
    uint32_t* pw = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
    for (int c = 0; c < 4; ++c) pw[c] = pack_bf16(acc[2 * c] * inv, acc[2 * c + 1] * inv);
    *reinterpret_cast<uint4*>(orow) = packed;
}

}  // namespace cb200
