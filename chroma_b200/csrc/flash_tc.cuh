// Flash attention for prefill chunks on the 5th-generation tensor cores (head_dim 64, bf16): the same sink attention
// as k_flash_prefill (chroma/models/gpt_oss.py:133-151, chroma/models/cached.py:36-47), with both products issued
// as tcgen05.mma into TMEM instead of mma.sync into registers.
//
// One CTA = two tiles of 128 query rows (256 consecutive rows) of one head of one sequence, which share every K and
// V tile; 10 warps:
//   warp 0 (one thread)  TMA: both Q tiles once, then K and V tiles of 64 keys into a 2-stage ring, plus each tile's
//                        key positions (ring slots or chunk rows) written by the warp's lanes
//   warp 1 (one thread)  allocates 256 TMEM columns (S of query tile k at [64k, 64k + 64), O of query tile k at
//                        [128 + 64k, ...)) and issues, per key tile t, in ping-pong order:
//                          O0 += P0(t).V(t), S0(t+1) = Q0.K(t+1), O1 += P1(t).V(t), S1(t+1) = Q1.K(t+1)
//                        (M=128, N=64, K=64 each; V read MN-major straight from its [key][dim] tile), each product
//                        as soon as the softmax of that query tile has written its P
//   warps 2-5, 6-9       the online softmax of query tile 0 and 1, one query row per thread (TMEM lane = row): load
//                        the S row, mask, running max in the log2 domain, rescale the O row in TMEM when the max
//                        grows, P = 2^(s - m) as bf16 into shared memory (the 128-byte-swizzled layout the MMA reads),
//                        running sum; at the end O / (sum + sink term), stored as bf16
// While one warpgroup works on its softmax, the tensor core runs the other tile's products: the exponentials and the
// MMAs overlap instead of alternating. Tiles with no visible key are never loaded (ring tiles screened against the
// slot positions, own tiles from the window's edge), as in k_flash_prefill. 2 CTAs fit an SM (100 KB shared memory,
// 256 TMEM columns each). All waits are bounded (tma.cuh).
#pragma once

#include "flash.cuh"
#include "tcgen05.cuh"

namespace cb200 {

constexpr int kFtRows = 128;  // query rows per query tile
constexpr int kFtQ = 2;       // query tiles per CTA
constexpr int kFtKeys = 64;   // keys per tile
constexpr int kFtThreads = 320;
constexpr int kFtMaxCacheTiles = 1024;
constexpr int kFtTile = kFtKeys * kFaDim * 2;  // one K or V tile: 8 KB
// Q 2 x 16 KB | K,V x 2 stages 32 KB | P 2 x 16 KB | key positions 1 KB | live cache tiles 2 KB + bits 128 B, + alignment
constexpr size_t kFtSmemBytes = 1024 + kFtQ * kFtRows * kFaDim * 2 + 4 * size_t(kFtTile) + kFtQ * kFtRows * kFtKeys * 2 +
                                2 * kFtKeys * sizeof(int64_t) + kFtMaxCacheTiles * 2 + kFtMaxCacheTiles / 8;

struct FlashMaps {
    CUtensorMap q;       // [B*n][H][64]: box {64, 1, 128}
    CUtensorMap kn, vn;  // chunk rows [B*n][KV][64]: box {64, 1, 64}
    CUtensorMap kc, vc;  // ring cache of this layer [B][ctx][KV][64] (4-D): box {64, 1, 64, 1}
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}
// Generic-proxy shared-memory writes (P) made visible to the tensor cores' async proxy.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Shared-memory descriptor of a 128-byte-swizzled tile read MN-major (rows of 64 elements along N, 8-row atoms of
// 1024 bytes along K): the V tile [key][dim] as the B operand of P.V.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(const void* smem_tile) {
    const uint64_t addr = smem_addr(smem_tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;
    d |= uint64_t(8192 >> 4) << 16;   // LBO: next 64-element block along N (a single block here)
    d |= uint64_t(1024 >> 4) << 32;   // SBO: next 8 keys
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

__device__ __forceinline__ void tmem_store32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// grid = (ceil(n / 256), H, B); block = kFtThreads; dynamic shared memory kFtSmemBytes.
__global__ void __launch_bounds__(kFtThreads, 2) k_flash_prefill_tc(const __grid_constant__ FlashMaps maps, FlashArgs a,
                                                                    const __nv_bfloat16* __restrict__ sinks,
                                                                    __nv_bfloat16* __restrict__ out, unsigned* err) {
    extern __shared__ uint8_t ft_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ft_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm;                                      // [2][128][64] SW128
    uint8_t* KV = Qs + kFtQ * kFtRows * kFaDim * 2;        // stage s: K at KV + 2s*tile, V at KV + (2s+1)*tile
    uint8_t* Ps = KV + 4 * kFtTile;                        // [2][128][64] SW128
    int64_t* tpos = reinterpret_cast<int64_t*>(Ps + kFtQ * kFtRows * kFtKeys * 2);  // [2][64] key positions
    uint16_t* live_list = reinterpret_cast<uint16_t*>(tpos + 2 * kFtKeys);
    uint32_t* live_bits = reinterpret_cast<uint32_t*>(live_list + kFtMaxCacheTiles);
    __shared__ uint64_t q_full, kv_full[2], kv_empty[2], s_full[kFtQ], p_full[kFtQ], pv_done[kFtQ];
    __shared__ uint32_t tmem_base;
    __shared__ int s_nlive;
    __shared__ volatile int abort_flag;

    const int qb = gridDim.x - 1 - blockIdx.x;  // heavy (late) query blocks first
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / a.G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i0 = qb * kFtQ * kFtRows;
    const int i_last = min(i0 + kFtQ * kFtRows, a.n) - 1;
    const int cache_tiles = (a.ctx + kFtKeys - 1) / kFtKeys;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int k = 0; k < kFtQ; ++k) {
            mbar_init(&s_full[k], 1);
            mbar_init(&p_full[k], 4);  // the 4 softmax warps of query tile k
            mbar_init(&pv_done[k], 1);
        }
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&maps.q);
        prefetch_tensormap(&maps.kn);
        prefetch_tensormap(&maps.vn);
        if (a.ctx) {
            prefetch_tensormap(&maps.kc);
            prefetch_tensormap(&maps.vc);
        }
    }
    for (int w = threadIdx.x; w < (cache_tiles + 31) / 32; w += blockDim.x) live_bits[w] = 0;
    if (warp == 1) {
        tmem_alloc(&tmem_base, 256);
        tmem_relinquish();
    }
    pdl_wait();
    pdl_trigger();
    const int64_t p0 = a.pos0 ? a.pos0[b] : 0;
    const int64_t first = p0 + i0, last = p0 + i_last;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Screen the ring: a cache tile is live when one of its slots holds a position some row of the block can see.
    for (int j = threadIdx.x; j < a.ctx; j += blockDim.x) {
        const int64_t tj = a.slots[size_t(b) * a.ctx + j];
        if (tj >= 0 && tj <= last && (a.window <= 0 || tj > first - a.window))
            atomicOr(&live_bits[(j / kFtKeys) >> 5], 1u << ((j / kFtKeys) & 31));
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
    const int own_lo = a.window > 0 ? max(0, i0 - a.window + 1) / kFtKeys : 0;
    const int own_hi = (i_last + kFtKeys) / kFtKeys;
    const int tiles = nlive + max(0, own_hi - own_lo);
    const uint32_t tmem = tmem_base;
    auto tile_key0 = [&](int tile, bool& cached) {
        cached = tile < nlive;
        return (cached ? int(live_list[tile]) : own_lo + tile - nlive) * kFtKeys;
    };

    if (warp == 0) {
        // ---- producer: both Q tiles once, then K/V tiles and their key positions
        if (lane == 0) {
            mbar_arrive_expect_tx(&q_full, kFtQ * kFtRows * kFaDim * 2);
            for (int k = 0; k < kFtQ; ++k)
                tma_load_3d(Qs + size_t(k) * kFtRows * kFaDim * 2, &maps.q, 0, h, b * a.n + i0 + k * kFtRows, &q_full);
        }
        for (int t = 0; t < tiles && !abort_flag; ++t) {
            const int s = t & 1;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&kv_empty[s], unsigned(((t >> 1) & 1) ^ 1), err);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) {
                if (lane == 0) abort_flag = 1;
                break;
            }
            bool cached;
            const int j0 = tile_key0(t, cached);
            const int limit = cached ? a.ctx : a.n;
            for (int c = lane; c < kFtKeys; c += 32) {
                const int j = j0 + c;
                tpos[s * kFtKeys + c] = j < limit ? (cached ? a.slots[size_t(b) * a.ctx + j] : p0 + j) : -1;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&kv_full[s], 2 * kFtTile);
                uint8_t* Kd = KV + size_t(2 * s) * kFtTile;
                uint8_t* Vd = KV + size_t(2 * s + 1) * kFtTile;
                if (cached) {
                    tma_load_4d(Kd, &maps.kc, 0, kvh, j0, b, &kv_full[s]);
                    tma_load_4d(Vd, &maps.vc, 0, kvh, j0, b, &kv_full[s]);
                } else {
                    tma_load_3d(Kd, &maps.kn, 0, kvh, b * a.n + j0, &kv_full[s]);
                    tma_load_3d(Vd, &maps.vn, 0, kvh, b * a.n + j0, &kv_full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue, ping-pong over the two query tiles
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc_bf16(kFtRows, kFtKeys);
            constexpr uint32_t idesc_o = umma_idesc_bf16(kFtRows, kFaDim) | (1u << 16);  // B (V) MN-major
            if (!mbar_wait(&q_full, 0, err)) abort_flag = 1;
            tc_fence_after();
            // S_k(u) = Q_k . K(u) into query tile k's S columns (K of tile u has landed: waited by the caller).
            auto issue_s = [&](int k, int u) {
                const uint64_t dq = umma_desc_sw128(Qs + size_t(k) * kFtRows * kFaDim * 2);
                const uint64_t dk = umma_desc_sw128(KV + size_t(2 * (u & 1)) * kFtTile);
#pragma unroll
                for (int kk = 0; kk < kFaDim / 16; ++kk)
                    umma_bf16(tmem + uint32_t(k * kFtKeys), dq + 2 * kk, dk + 2 * kk, idesc_s, kk > 0);
                umma_commit(&s_full[k]);
            };
            auto wait_kv = [&](int u) {
                if (!mbar_wait(&kv_full[u & 1], unsigned((u >> 1) & 1), err)) return false;
                tc_fence_after();
                return true;
            };
            if (tiles > 0 && !abort_flag) {
                if (wait_kv(0)) {
                    issue_s(0, 0);
                    issue_s(1, 0);
                } else {
                    abort_flag = 1;
                }
            }
            for (int t = 0; t < tiles && !abort_flag; ++t) {
                const int s = t & 1;
                const uint64_t dv = umma_desc_sw128_mn(KV + size_t(2 * s + 1) * kFtTile);
                bool next_ready = false;
                for (int k = 0; k < kFtQ; ++k) {
                    // Query tile k's softmax has written P_k(t) (and finished reading S_k(t)).
                    if (!mbar_wait(&p_full[k], unsigned(t & 1), err)) { abort_flag = 1; break; }
                    tc_fence_after();
                    const uint64_t dp = umma_desc_sw128(Ps + size_t(k) * kFtRows * kFtKeys * 2);
                    const uint32_t tO = tmem + uint32_t(2 * kFtKeys + k * kFaDim);
#pragma unroll
                    for (int kk = 0; kk < kFtKeys / 16; ++kk)  // 16 keys per step: +32 B along P's rows, +2 KB down V
                        umma_bf16(tO, dp + 2 * kk, dv + 128 * kk, idesc_o, t > 0 || kk > 0);
                    umma_commit(&pv_done[k]);
                    if (k == kFtQ - 1) umma_commit(&kv_empty[s]);
                    if (t + 1 < tiles) {
                        if (k == 0) {
                            if (!wait_kv(t + 1)) { abort_flag = 1; break; }
                            next_ready = true;
                        }
                        if (next_ready) issue_s(k, t + 1);
                    }
                }
            }
        }
    } else {
        // ---- softmax of query tile k: warp q (= warp % 4) owns TMEM lanes / tile rows [32q, 32q + 32)
        const int k = (warp - 2) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;  // this thread's query row within its tile
        const int i = i0 + k * kFtRows + r;
        const int ik0 = i0 + k * kFtRows, ik_last = min(ik0 + kFtRows, a.n) - 1;
        const int64_t ti = p0 + i;
        const bool row_ok = i < a.n;
        const uint32_t lane_base = uint32_t(q * 32) << 16;
        const uint32_t tS = tmem + uint32_t(k * kFtKeys) + lane_base;
        const uint32_t tO = tmem + uint32_t(2 * kFtKeys + k * kFaDim) + lane_base;
        uint8_t* prow = Ps + size_t(k) * kFtRows * kFtKeys * 2 + size_t(r) * 128;
        float m_run = -INFINITY, l_run = 0.f;
        for (int t = 0; t < tiles && !abort_flag; ++t) {
            const int s = t & 1;
            bool cached;
            const int j0 = tile_key0(t, cached);
            if (!mbar_wait(&kv_full[s], unsigned((t >> 1) & 1), err) || !mbar_wait(&s_full[k], unsigned(t & 1), err)) {
                abort_flag = 1;
                break;
            }
            tc_fence_after();
            const bool masked = cached || j0 + kFtKeys - 1 > ik0 || (a.window > 0 && j0 <= ik_last - a.window);
            // Two passes over the S row (32 columns at a time keeps the registers low): the max, then P.
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                float v[32];
                tmem_load32(tS + c * 32, v);
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    if (masked) {
                        const int64_t tj = tpos[s * kFtKeys + c * 32 + e];
                        if (!(row_ok && tj >= 0 && tj <= ti && (a.window <= 0 || tj > ti - a.window))) v[e] = -INFINITY;
                    }
                    mx = fmaxf(mx, v[e]);
                }
            }
            // Lazy rescaling: the reference max moves only when the tile's max exceeds it by more than 8 (log2
            // domain), so P stays below 2^8 and most tiles leave O untouched; the sum uses the same reference, so the
            // result is unchanged.
            const float m_tile = mx * a.scale_log2;
            const float m_new = (m_run == -INFINITY || m_tile > m_run + 8.f) ? fmaxf(m_run, m_tile) : m_run;
            const bool none = m_new == -INFINITY;
            const float corr = none ? 1.f : fast_exp2(m_run - m_new);
            const float neg = none ? 0.f : -m_new;
            // The previous P_k.V must have finished before O_k is rescaled and P_k is overwritten.
            if (t > 0) {
                if (!mbar_wait(&pv_done[k], unsigned((t - 1) & 1), err)) { abort_flag = 1; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
                    for (int c = 0; c < 2; ++c) {
                        float ov[32];
                        tmem_load32(tO + c * 32, ov);
#pragma unroll
                        for (int e = 0; e < 32; ++e) ov[e] *= corr;
                        tmem_store32(tO + c * 32, ov);
                    }
                }
            }
            float rs = 0.f;
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
                float v[32];
                tmem_load32(tS + c * 32, v);
#pragma unroll
                for (int cc = 0; cc < 4; ++cc) {  // 16-byte chunk ch = 4c + cc of the row (keys 8ch..8ch+7), swizzled
                    uint32_t w4[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = cc * 8 + 2 * u;
                        float pa = 0.f, pb = 0.f;
                        bool va = true, vb = true;
                        if (masked) {
                            const int64_t ta = tpos[s * kFtKeys + c * 32 + e], tb = tpos[s * kFtKeys + c * 32 + e + 1];
                            va = row_ok && ta >= 0 && ta <= ti && (a.window <= 0 || ta > ti - a.window);
                            vb = row_ok && tb >= 0 && tb <= ti && (a.window <= 0 || tb > ti - a.window);
                        }
                        if (va) pa = fast_exp2(fmaf(v[e], a.scale_log2, neg));
                        if (vb) pb = fast_exp2(fmaf(v[e + 1], a.scale_log2, neg));
                        rs += pa + pb;
                        w4[u] = pack_bf16(pa, pb);
                    }
                    const int ch = 4 * c + cc;
                    *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
            l_run = l_run * corr + rs;
            m_run = m_new;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[k]);
        }
        // Final: wait for the last P_k.V, then O / (l + sink term) for this row.
        if (tiles > 0 && !abort_flag && mbar_wait(&pv_done[k], unsigned((tiles - 1) & 1), err)) {
            tc_fence_after();
            float ov[2][32];
            tmem_load32(tO, ov[0]);
            tmem_load32(tO + 32, ov[1]);
            if (row_ok) {
                const float sink = __bfloat162float(sinks[h]) * 1.4426950408889634f;
                const float mf = fmaxf(m_run, sink);
                const float c = m_run == -INFINITY ? 0.f : exp2f(m_run - mf);
                const float inv = 1.0f / (l_run * c + exp2f(sink - mf));
                __nv_bfloat16* orow = out + ((size_t(b) * a.n + i) * a.H + h) * kFaDim;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    uint32_t w4[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = ch * 8 + 2 * u;
                        w4[u] = pack_bf16(ov[e >> 5][e & 31] * c * inv, ov[(e + 1) >> 5][(e + 1) & 31] * c * inv);
                    }
                    *reinterpret_cast<uint4*>(orow + ch * 8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

}  // namespace cb200
