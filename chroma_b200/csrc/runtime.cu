// chroma_b200 runtime: the C ABI of include/chroma_b200.h.
//
// Replaces the reference's header-only CUDA runtime (chroma/_src/codegen/cuda/runtime.h:89-201) and the generated
// per-graph launch list (chroma/_src/codegen/cuda/codegen.py:13-41, :87-111). Differences by design:
//   * kernels are precompiled for sm_100a (no per-graph nvcc); a program is a descriptor + weights file;
//   * one call's kernel sequence is captured once into a CUDA graph and replayed; kernels use programmatic
//     dependent launch so each one's prologue (weight prefetch) overlaps its predecessor's tail;
//   * device weights are shared between programs loaded from identical weight files (prefill/decode pairs);
//   * KV-cached decoding can keep the cache in device memory (chroma_b200_decoder_*).
// Error contract kept from the reference: an out-of-range index sets a device error word, the call finishes,
// synchronises and reports CHROMA_B200_INDEX (IndexError); the program stays usable (runtime.h:147-173).

#include "../../include/chroma_b200.h"
#include "flash.cuh"
#include "flash_tc.cuh"
#include "decode_cluster.cuh"
#include "fwd_cluster.cuh"
#include "ep.cuh"
#include "gemm.cuh"
#include "gptoss.cuh"
#include "large.cuh"
#include "micro.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <array>
#include <type_traits>
#include <vector>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace cb200 {

struct IndexError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct ValueError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

static void check(cudaError_t st, const char* what) {
    if (st != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(st));
}

class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        check(cudaGetDevice(&previous_), "cudaGetDevice");
        if (previous_ != device) check(cudaSetDevice(device), "cudaSetDevice");
        device_ = device;
    }
    ~DeviceGuard() {
        if (previous_ != device_) cudaSetDevice(previous_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int previous_ = 0, device_ = 0;
};

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    explicit DevBuf(size_t n) : bytes(n) { check(cudaMalloc(&p, n ? n : 1), "cudaMalloc"); }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        std::swap(p, o.p);
        std::swap(bytes, o.bytes);
        return *this;
    }
    template <typename T> T* as() const { return static_cast<T*>(p); }
};

struct PinnedBuf {
    void* p = nullptr;
    explicit PinnedBuf(size_t n) { check(cudaMallocHost(&p, n ? n : 1), "cudaMallocHost"); }
    ~PinnedBuf() {
        if (p) cudaFreeHost(p);
    }
    PinnedBuf(const PinnedBuf&) = delete;
    PinnedBuf& operator=(const PinnedBuf&) = delete;
};

// ---------------------------------------------------------------------------------------------------------
// Weights: read once per (device, file identity) and shared by every program that names the same file.
struct Weights {
    int device;
    DevBuf buf;           // owned copy of a weights file
    const char* ptr = nullptr;  // device address of the weights (owned buffer or caller-owned memory)
};

static std::mutex g_weights_mu;
static std::map<std::string, std::weak_ptr<Weights>> g_weights;

static std::shared_ptr<Weights> load_weights(const char* path, size_t bytes, int device) {
    std::string p(path);
    const std::string base = p.substr(p.find_last_of('/') == std::string::npos ? 0 : p.find_last_of('/') + 1);
    const std::string key = std::to_string(device) + ":" + base + ":" + std::to_string(bytes);
    std::lock_guard<std::mutex> lock(g_weights_mu);
    auto it = g_weights.find(key);
    if (it != g_weights.end()) {
        if (auto live = it->second.lock()) return live;
    }
    std::ifstream stream(p, std::ios::binary | std::ios::ate);
    if (!stream || stream.tellg() != static_cast<std::streamoff>(bytes))
        throw std::runtime_error("Missing weights file or incorrect byte size");
    stream.seekg(0);
    auto w = std::make_shared<Weights>();
    w->device = device;
    w->buf = DevBuf(bytes);
    // Upload through a pinned bounce buffer in 64 MiB pieces.
    const size_t piece = size_t(64) << 20;
    PinnedBuf stage(std::min(bytes, piece));
    for (size_t off = 0; off < bytes; off += piece) {
        const size_t n = std::min(piece, bytes - off);
        if (!stream.read(static_cast<char*>(stage.p), static_cast<std::streamsize>(n)))
            throw std::runtime_error("Cannot read weights");
        check(cudaMemcpy(w->buf.as<char>() + off, stage.p, n, cudaMemcpyHostToDevice), "Upload weights");
    }
    w->ptr = w->buf.as<const char>();
    g_weights[key] = w;
    return w;
}

// ---------------------------------------------------------------------------------------------------------
// Kernel launch with programmatic stream serialisation (PDL).
template <typename... Params, typename... Args>
static void launch(cudaStream_t s, dim3 grid, dim3 block, size_t smem, void (*kernel)(Params...), Args&&... args) {
    if (smem > 48 * 1024)
        check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "smem attribute");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...), "kernel launch");
}

// Launch configuration of a kernel run as thread-block clusters of `cluster` CTAs (sizes above 8 are opted in),
// with programmatic dependent launch like launch().
struct ClusterLaunch {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    template <typename... Params>
    ClusterLaunch(cudaStream_t s, dim3 grid, dim3 block, size_t smem, int cluster, void (*kernel)(Params...)) {
        check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)), "smem attribute");
        if (cluster > 8) check(cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                               "cluster size attribute");
        cfg.gridDim = grid;
        cfg.blockDim = block;
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = unsigned(cluster);
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
    }
};

// ---------------------------------------------------------------------------------------------------------
// TMA tensor maps. cuTensorMapEncodeTiled is a driver entry point, fetched at run time (no link against libcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q), "cuTensorMapEncodeTiled");
        if (!p || q != cudaDriverEntryPointSuccess) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Row-major bf16 matrix [rows][cols] read in boxes of box_rows x 64 columns with the 128-byte swizzle.
static CUtensorMap bf16_tile_map(const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    if (reinterpret_cast<uintptr_t>(base) % 16 || (cols * 2) % 16)
        throw ValueError("TMA operands need 16-byte aligned bases and rows");
    CUtensorMap map;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {uint32_t(kGemmBK), box_rows};
    const cuuint32_t elem[2] = {1, 1};
    const CUresult r = encode_tiled()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                                      elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
    return map;
}

// bf16 tensor of rank 3 or 4 (dims innermost first, byte strides of dims 1..rank-1) read in boxes with the 128-byte
// swizzle; the innermost box is 64 elements (one 128-byte row).
static CUtensorMap bf16_map_nd(const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                               const uint32_t* box) {
    if (reinterpret_cast<uintptr_t>(base) % 16) throw ValueError("TMA operands need 16-byte aligned bases");
    for (int i = 0; i < rank - 1; ++i)
        if (strides[i] % 16) throw ValueError("TMA strides must be multiples of 16 bytes");
    CUtensorMap map;
    cuuint64_t d[5];
    cuuint64_t st[4];
    cuuint32_t bx[5], el[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
        el[i] = 1;
    }
    for (int i = 0; i < rank - 1; ++i) st[i] = strides[i];
    const CUresult res = encode_tiled()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, cuuint32_t(rank), const_cast<void*>(base), d,
                                        st, bx, el, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (res != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(res)));
    return map;
}

// C = A . B^T on the tensor cores. Dense when groups == 1 and offsets == nullptr; grouped otherwise (offsets and
// offsets is a device array of groups + 1 ints; tile_scratch is unused).
// Split-K factor for a dense GEMM that would leave most SMs idle (decode-sized M): enough splits to give every SM a
// tile, at least 4 K blocks per split, at most 8 splits.
static int splitk_choice(int M, int N, int K, int bn, int sms) {
    const int tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + bn - 1) / bn);
    const int kblocks = (K + kGemmBK - 1) / kGemmBK;
    if (tiles * 2 > sms) return 1;
    const int k = std::min({8, sms / std::max(1, tiles), kblocks / 4});
    return k >= 2 ? k : 1;
}

static void gemm_bf16(cudaStream_t s, const void* A, const void* B, GemmArgs g, int rows_a, int rows_b, void* tile_scratch,
                      int sms, unsigned* err, float* splitk_ws = nullptr, size_t splitk_ws_bytes = 0) {
    if (g.groups < 1 || g.groups > kGemmMaxGroups) throw ValueError("GEMM group count out of range");
    if (g.K % 8) throw ValueError("GEMM K must be a multiple of 8");
    if (g.epi == kEpiSwiglu && g.N % 32) throw ValueError("SwiGLU epilogue needs N a multiple of 32");
    const bool narrow = g.N <= 32;
    if (g.epi == kEpiRope && (narrow || g.N % 64 || g.ldc % 8 || g.rope_KV < 1 || g.offsets ||
                              ((reinterpret_cast<uintptr_t>(g.C) | reinterpret_cast<uintptr_t>(g.rope_k) |
                                reinterpret_cast<uintptr_t>(g.rope_v) | reinterpret_cast<uintptr_t>(g.bias) |
                                reinterpret_cast<uintptr_t>(g.rope_cs)) & 15)))
        throw ValueError("RoPE epilogue needs whole 64-wide heads, a dense GEMM and 16-byte aligned outputs");
    const CUtensorMap ma = bf16_tile_map(A, uint64_t(rows_a), uint64_t(g.K), kGemmBM);
    // The CTA-pair kernel (256 x 256 tiles over two SMs, two thirds of the operand bytes per SM) measured faster only
    // for the grouped SwiGLU GEMM of the prefill MoE (0.93 vs 0.99 ms at 32,768 x 5,760 x 2,880); the single-CTA
    // kernel wins the dense and expert-down shapes. CHROMA_B200_PAIR_GEMM=0/1 forces it off/on where it applies.
    static const char* pair_env = std::getenv("CHROMA_B200_PAIR_GEMM");
    const bool pair_auto = g.offsets && g.epi == kEpiSwiglu && rows_a >= 8192;
    const bool pair_on = pair_env ? pair_env[0] == '1' : pair_auto;
    if (pair_on && !narrow && sms >= 2 && g.epi != kEpiRope) {
        const int pair_tiles = g.offsets ? sms : ((g.M + kPairBM - 1) / kPairBM) * ((g.N + kPairBN - 1) / kPairBN);
        if (g.offsets ? rows_a >= 8192 : (g.M >= 1024 && pair_tiles * 2 >= sms)) {
            const CUtensorMap mb2 = bf16_tile_map(B, uint64_t(rows_b), uint64_t(g.K), 128);
            g.ksplit = 1;
            const dim3 grid(unsigned(2 * std::max(1, std::min(pair_tiles, sms / 2))));
            launch(s, grid, dim3(kGemmThreads), kPairSmemBytes, k_gemm_bf16_pair, ma, mb2, g, err);
            return;
        }
    }
    const CUtensorMap mb = bf16_tile_map(B, uint64_t(rows_b), uint64_t(g.K), narrow ? 32 : 256);
    (void)tile_scratch;  // tile prefix sums are computed in the kernel's prologue
    const int bn = narrow ? 32 : 256;
    // A last column tile of at most 128 columns (N = 2,880: 64) runs as a narrow MMA after the full-width tiles
    // (GemmArgs::tail_n). CHROMA_B200_GEMM_TAIL=0 keeps it at full width.
    static const char* tail_env = std::getenv("CHROMA_B200_GEMM_TAIL");
    const int ntiles_n = (g.N + bn - 1) / bn, tail_w = g.N - (ntiles_n - 1) * bn;
    g.tail_n = !narrow && ntiles_n >= 2 && tail_w <= 128 && !(tail_env && tail_env[0] == '0') ? (tail_w + 15) / 16 * 16 : 0;
    const CUtensorMap mbt = g.tail_n ? bf16_tile_map(B, uint64_t(rows_b), uint64_t(g.K), g.tail_n) : mb;
    int tiles = g.offsets ? sms : ((g.M + kGemmBM - 1) / kGemmBM) * ((g.N + bn - 1) / bn);
    g.ksplit = 1;
    if (!g.offsets && splitk_ws && (g.epi == kEpiStore || g.epi == kEpiResidual)) {
        const int k = splitk_choice(g.M, g.N, g.K, bn, sms);
        if (k > 1 && size_t(k) * g.M * g.N * 4 <= splitk_ws_bytes) {
            g.ksplit = k;
            g.partial = splitk_ws;
            tiles *= k;
        }
    }
    const dim3 grid(unsigned(std::max(1, std::min(tiles, sms))));
    const size_t smem = size_t(kGemmStages) * (kGemmBM + bn) * kGemmBK * 2 + 4 * kGemmStageBytes + 1024;
    if (narrow) launch(s, grid, dim3(kGemmThreads), smem, k_gemm_bf16<32>, ma, mb, mbt, g, err);
    else launch(s, grid, dim3(kGemmThreads), smem, k_gemm_bf16<256>, ma, mb, mbt, g, err);
    if (g.ksplit > 1)
        launch(s, dim3(unsigned((g.N + 511) / 512), unsigned(g.M)), dim3(256), 0, k_gemm_splitk_epilogue, g);
}

// ---------------------------------------------------------------------------------------------------------
// Small utility kernels.
__global__ void k_positions(const int64_t* pos0, int B, int n, float* positions, int64_t* last, int count,
                            unsigned* err) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0 && err) *err = 0u;  // the step's error word starts clear
    if (i < B * n) positions[i] = float(pos0[i / n] + i % n);
    if (i < B) last[i] = count - 1;
}

template <typename T>
__global__ void k_commit(const T* new_k, const T* new_v, int L, int B, int n, int count, int ctx, int KV, int hd,
                         const int64_t* pos0, T* cache_k, T* cache_v, int64_t* slots) {
    pdl_wait();
    pdl_trigger();
    // One block per (layer, sequence, row < count); threads over KV*hd.
    const int r = blockIdx.x % count;
    const int b = (blockIdx.x / count) % B;
    const int l = blockIdx.x / (count * B);
    const int64_t t = pos0[b] + r;
    const int slot = int(t % ctx);
    const size_t row = size_t(KV) * hd;
    const T* sk = new_k + (size_t(l) * B * n + size_t(b) * n + r) * row;
    const T* sv = new_v + (size_t(l) * B * n + size_t(b) * n + r) * row;
    T* dk = cache_k + ((size_t(b) * L + l) * ctx + slot) * row;
    T* dv = cache_v + ((size_t(b) * L + l) * ctx + slot) * row;
    for (size_t i = threadIdx.x; i < row; i += blockDim.x) {
        dk[i] = sk[i];
        dv[i] = sv[i];
    }
    if (l == 0 && threadIdx.x == 0) slots[size_t(b) * ctx + slot] = t;
}

// After a device-only greedy step: feed each sequence's argmax back as its next token, advance its position and
// append the id to the generation record.
__global__ void k_advance(const unsigned long long* keys, int B, int64_t* tokens, int64_t* pos0, int64_t* record,
                          int* counter, int capacity) {
    pdl_wait();
    pdl_trigger();
    const int step = *counter;
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        const int64_t id = argmax_index(keys[b]);
        tokens[b] = id;
        pos0[b] += 1;
        if (step < capacity) record[size_t(step) * B + b] = id;
    }
    __syncthreads();
    if (threadIdx.x == 0) *counter = step + 1;
}

// Vocab GEMV launch: the row-count template is the smallest that covers `rows` (a decode step has one row), and the
// grid is exactly the CTAs that fit on the GPU at once (one wave of a grid-stride loop).
template <typename T, int R>
static void launch_vocab_r(cudaStream_t s, const Dims& dm, int sms, const float* x, int rows, const T* W, T* logits,
                           unsigned long long* keys) {
    const size_t smem = size_t(R) * dm.d * 4;
    int per_sm = 0;
    check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_vocab<T, R>, kThreads, smem), "vocab occupancy");
    const int vgrid = std::max(1, std::min((dm.V + 31) / 32, sms * std::max(1, per_sm)));
    launch(s, dim3(vgrid), dim3(kThreads), smem, k_vocab<T, R>, x, rows, dm.d, dm.V, W, logits, keys);
}

template <typename T, int R>
static void launch_vocab_tma(cudaStream_t s, const Dims& dm, int sms, const float* x, int rows, const T* W, T* logits,
                             unsigned long long* keys, unsigned* err) {
    const int row_bytes = dm.d * int(sizeof(T));
    const int rb = kVocabStageBytes / row_bytes;
    const size_t smem = size_t(kVocabStages) * kVocabStageBytes + size_t(R) * dm.d * 4;
    const int nblocks = (dm.V + rb - 1) / rb;
    launch(s, dim3(std::min(nblocks, sms)), dim3(kThreads + 32), smem, k_vocab_tma<T, R>, x, rows, dm.d, dm.V, W, logits,
           keys, rb, err);
}

// Rows of at most 2 KiB that tile 32 KiB stages exactly go through the TMA-pipelined kernel; others (large hidden
// sizes) through the register-fragment kernel.
static bool vocab_tma_ok(const Dims& dm, size_t es) {
    const size_t row = size_t(dm.d) * es;
    return row % 16 == 0 && row <= 2048 && kVocabStageBytes % row == 0;
}

template <typename T>
static void launch_vocab(cudaStream_t s, const Dims& dm, int sms, const float* x, int rows, const T* W, T* logits,
                         unsigned long long* keys, unsigned* err, bool allow_tma = true) {
    // The TMA ring measured slower than the register-fragment kernel for the dev vocab (26.7 vs 21.6 us per launch,
    // same 103 MB of DRAM reads), so it is only selected when CHROMA_B200_VOCAB_TMA is set. Callers that never read
    // the program's error word (where the TMA ring reports a timed-out wait) pass allow_tma = false.
    static const bool use_tma = std::getenv("CHROMA_B200_VOCAB_TMA") != nullptr;
    if (allow_tma && use_tma && vocab_tma_ok(dm, sizeof(T)) && rows <= kVocabRows) {
        if (rows == 1) launch_vocab_tma<T, 1>(s, dm, sms, x, rows, W, logits, keys, err);
        else if (rows <= 2) launch_vocab_tma<T, 2>(s, dm, sms, x, rows, W, logits, keys, err);
        else if (rows <= 4) launch_vocab_tma<T, 4>(s, dm, sms, x, rows, W, logits, keys, err);
        else launch_vocab_tma<T, kVocabRows>(s, dm, sms, x, rows, W, logits, keys, err);
        return;
    }
    if constexpr (std::is_same_v<T, float>) {
        if (rows == 1 && dm.d == 128) {  // one decode row: balanced contiguous ranges (k_vocab_row)
            static int per_sm = 0;
            if (!per_sm) check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_vocab_row, kVrThreads, 0),
                               "vocab occupancy");
            const int grid = std::max(1, sms * std::max(1, per_sm) * 2);
            const int step = 4 * kVrU;
            const int rows_per_cta = ((dm.V + grid - 1) / grid + step - 1) / step * step;
            launch(s, dim3((dm.V + rows_per_cta - 1) / rows_per_cta), dim3(kVrThreads), 0, k_vocab_row, x, dm.V, W,
                   logits, keys, rows_per_cta);
            return;
        }
        if (rows > kVocabRows && dm.d == kVtD) {  // many rows: one pass over the vocab matrix per 64 rows
            const int tiles = (dm.V + kVtVocab - 1) / kVtVocab;
            launch(s, dim3(std::min(tiles, sms)), dim3(kThreads), kVtSmemBytes, k_vocab_tiled, x, rows, dm.V, W, logits,
                   keys);
            return;
        }
    }
    if (rows == 1) launch_vocab_r<T, 1>(s, dm, sms, x, rows, W, logits, keys);
    else if (rows <= 2) launch_vocab_r<T, 2>(s, dm, sms, x, rows, W, logits, keys);
    else if (rows <= 4) launch_vocab_r<T, 4>(s, dm, sms, x, rows, W, logits, keys);
    else launch_vocab_r<T, kVocabRows>(s, dm, sms, x, rows, W, logits, keys);
}

// ---------------------------------------------------------------------------------------------------------
// ---------------------------------------------------------------------------------------------------------
// Expert-parallel group: this rank's IPC-exported buffer (header, receive metadata, receive rows, return rows),
// the peers' buffers opened from their handles, and the rank-local epoch / last-CTA counters.
struct EpGroup {
    int rank = 0, world = 1, E = 0, d = 0, device = 0;
    long long pmax = 0, cap = 0;
    size_t off_meta = 0, off_x = 0, off_y = 0;
    int vrows_max = 0, V = 0, Vl = 0;  // vocab column shard (vrows_max == 0: off)
    size_t off_vrows = 0, off_vkeys = 0, off_vlogits = 0;
    int vocab_rows_here() const { return std::max(0, std::min(Vl, V - rank * Vl)); }
    DevBuf shared, local;
    std::array<char*, kEpMaxWorld> peer{};
    std::vector<void*> opened;
    bool open = false;
    unsigned long long timeout_ns = 10'000'000'000ull;  // CHROMA_B200_EP_TIMEOUT_MS overrides (read at creation)

    ~EpGroup() {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        cudaDeviceSynchronize();
        for (void* q : opened) cudaIpcCloseMemHandle(q);
        cudaSetDevice(prev);
    }

    EpArgs args(int El) const {
        EpArgs a{};
        a.rank = rank;
        a.world = world;
        a.E = E;
        a.El = El;
        a.d = d;
        a.pmax = pmax;
        a.cap = cap;
        for (int q = 0; q < kEpMaxWorld; ++q) a.peer[q] = peer[size_t(q)];
        a.off_meta = off_meta;
        a.off_x = off_x;
        a.off_y = off_y;
        a.epoch = local.as<unsigned>();
        a.done = local.as<unsigned>() + 1;
        a.timeout_ns = timeout_ns;
        a.vrows_max = vrows_max;
        a.V = V;
        a.Vl = Vl;
        a.off_vrows = off_vrows;
        a.off_vkeys = off_vkeys;
        a.off_vlogits = off_vlogits;
        return a;
    }
    __nv_bfloat16* recv_rows() const { return reinterpret_cast<__nv_bfloat16*>(shared.as<char>() + off_x); }
    __nv_bfloat16* return_rows() const { return reinterpret_cast<__nv_bfloat16*>(shared.as<char>() + off_y); }
};

struct Model {
    chroma_b200_desc desc{};
    std::shared_ptr<EpGroup> ep;  // expert-parallel group, or null (all experts local)
    int El = 0;                   // experts held by this program (E / world)
    Dims dm{};
    std::vector<int32_t> layer_window;
    std::vector<int64_t> offsets;
    std::shared_ptr<Weights> weights;
    DevBuf inv_freq;
    int device = 0;

    const char* at(int i) const { return weights->ptr + offsets.at(size_t(i)); }
    template <typename T> LayerW<T> layer(int l) const {
        const int b = 3 + 13 * l;
        LayerW<T> w;
        w.attn_norm = reinterpret_cast<const float*>(at(b + 0));
        w.sinks = reinterpret_cast<const T*>(at(b + 1));
        w.qkv_w = reinterpret_cast<const T*>(at(b + 2));
        w.qkv_b = reinterpret_cast<const T*>(at(b + 3));
        w.out_w = reinterpret_cast<const T*>(at(b + 4));
        w.out_b = reinterpret_cast<const T*>(at(b + 5));
        w.mlp_norm = reinterpret_cast<const float*>(at(b + 6));
        w.gate_w = reinterpret_cast<const T*>(at(b + 7));
        w.gate_b = reinterpret_cast<const T*>(at(b + 8));
        w.w1 = reinterpret_cast<const T*>(at(b + 9));
        w.b1 = reinterpret_cast<const T*>(at(b + 10));
        w.w2 = reinterpret_cast<const T*>(at(b + 11));
        w.b2 = reinterpret_cast<const T*>(at(b + 12));
        return w;
    }
};

static size_t storage_size(int storage) { return storage == CHROMA_B200_BF16 ? 2 : 4; }

static void validate_desc(const chroma_b200_desc& d) {
    auto need = [](bool ok, const char* what) {
        if (!ok) throw ValueError(std::string("invalid program descriptor: ") + what);
    };
    need(d.storage == CHROMA_B200_FP32 || d.storage == CHROMA_B200_BF16, "storage");
    need(d.offsets != nullptr && d.num_offsets > 0, "offsets");
    if (d.kind == CHROMA_B200_MICRO) {
        need(d.storage == CHROMA_B200_BF16, "micro storage");
        need(d.rows > 0 && d.rows < (int64_t(1) << 31) && d.cols > 0 && d.cols % 8 == 0 && d.cols <= 8 * 512 * 8, "micro shape");
        return;
    }
    need(d.kind == CHROMA_B200_GPTOSS_FORWARD || d.kind == CHROMA_B200_GPTOSS_CACHED || d.kind == CHROMA_B200_GPTOSS_LAST,
         "kind");
    need(d.layers > 0 && d.num_offsets == 3 + 13 * d.layers, "layer count / offsets");
    need(d.hidden > 0 && d.hidden % 4 == 0, "hidden size (multiple of 4)");
    need(d.heads > 0 && d.kv_heads > 0 && d.heads % d.kv_heads == 0 && d.heads / d.kv_heads <= 8, "heads (query groups of at most 8)");
    need(d.head_dim > 0 && d.head_dim % 4 == 0 && d.head_dim <= 64, "head_dim (multiple of 4, <= 64)");
    need(d.experts > 0 && d.experts <= 256 && d.top_k > 0 && d.top_k <= 8 && d.top_k <= d.experts, "experts");
    need(d.intermediate > 0 && d.intermediate % 4 == 0, "intermediate size");
    need(d.vocab > 0 && d.tokens > 0, "vocab / tokens");
    need(d.kind != CHROMA_B200_GPTOSS_CACHED || d.context > 0, "context");
    need(d.inv_freq != nullptr && d.layer_window != nullptr, "rope / window tables");
}

// ---------------------------------------------------------------------------------------------------------
// Arena planning: best fit over inclusive kernel-index lifetimes with a coalesced free list, the algorithm of the
// reference's planner (chroma/_src/memory.py:12-50). Visiting order is by start, ties in insertion order.
struct Alloc {
    size_t size;
    int start, end;
    size_t offset;
};

static size_t plan_arena(std::vector<Alloc>& allocs) {
    std::vector<size_t> order(allocs.size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return allocs[a].start < allocs[b].start; });
    std::vector<size_t> live;
    std::vector<std::pair<size_t, size_t>> free_list;  // (offset, size)
    size_t total = 0;
    for (size_t idx : order) {
        Alloc& a = allocs[idx];
        std::vector<size_t> still;
        for (size_t o : live) {
            if (allocs[o].end < a.start) free_list.emplace_back(allocs[o].offset, allocs[o].size);
            else still.push_back(o);
        }
        live.swap(still);
        std::sort(free_list.begin(), free_list.end());
        std::vector<std::pair<size_t, size_t>> merged;
        for (const auto& f : free_list) {
            if (!merged.empty() && merged.back().first + merged.back().second == f.first) merged.back().second += f.second;
            else merged.push_back(f);
        }
        free_list.swap(merged);
        long best = -1;
        for (size_t i = 0; i < free_list.size(); ++i)
            if (free_list[i].second >= a.size && (best < 0 || free_list[i].second < free_list[size_t(best)].second))
                best = long(i);
        if (best >= 0) {
            const auto f = free_list[size_t(best)];
            free_list.erase(free_list.begin() + best);
            a.offset = f.first;
            if (f.second > a.size) free_list.emplace_back(f.first + a.size, f.second - a.size);
        } else {
            a.offset = total;
            total += a.size;
        }
        live.push_back(idx);
    }
    return total;
}

// ---------------------------------------------------------------------------------------------------------
// One configured execution of a GPT-OSS model: B sequences of n rows, with its own activation arena.
struct GptIO {
    const int64_t* tokens = nullptr;
    const float* positions = nullptr;
    const void* cache_k = nullptr;  // [B][L][ctx][KV][hd]
    const void* cache_v = nullptr;
    void* new_k = nullptr;          // [L][B*n][KV][hd]
    void* new_v = nullptr;
    const void* mask = nullptr;     // [n][ctx+n] (buffer mode, B == 1)
    const void* window_mask = nullptr;
    const int64_t* slots = nullptr; // [B][ctx] (slots mode)
    const int64_t* pos0 = nullptr;  // [B]
    const int64_t* rows = nullptr;  // [B] selected row per sequence, or nullptr for every row
    void* logits = nullptr;
    unsigned long long* keys = nullptr;  // [rows] optional fused-argmax keys
    int* routes = nullptr;          // [L][B*n][k] optional record of the routing
    void* commit_k = nullptr;       // in-place commit of the new rows (device-resident decoding, cluster path)
    void* commit_v = nullptr;
    int64_t* commit_slots = nullptr;
};

// The large-width bf16 path (hidden >= 1024, head_dim 64): tensor-core GEMMs, flash attention for prefill chunks,
// expert grouping for the MoE. Used for the GPT-OSS-20B/120B shapes.
static bool is_large(const chroma_b200_desc& d) {
    return d.storage == CHROMA_B200_BF16 && d.hidden >= 1024 && d.hidden % 64 == 0 && d.head_dim == 64 &&
           d.intermediate % 64 == 0 && d.experts <= kGemmMaxGroups;
}

// Attention kernels at the large shapes: the TMA-staged ones (k_flash_prefill_tc on the tensor cores,
// k_flash_decode_tma) by default; CHROMA_B200_FLASH_TC=0 selects the cp.async / mma.sync pair (k_flash_prefill,
// k_flash_decode), kept as the cross-check. One C4 layer's prefill attention: 333 us against 705 us; one C5 layer's
// decode attention: 65 us against 78 us.
static bool tma_attention() {
    static const bool on = [] {
        const char* e = std::getenv("CHROMA_B200_FLASH_TC");
        return !(e && e[0] == '0');
    }();
    return on;
}

struct LargeExec {
    const Model* m = nullptr;
    int B = 1, n = 1, ctx = 0, mask_mode = kMaskBuffer, window = 0, sms = 148, chunks = 1, key_chunk = 256, rows = 1;
    int fd_splits = 1, fd_split_keys = 64;  // flash decoding: key splits per (sequence, KV head)
    float* fd_part = nullptr;
    DevBuf arena, counters, route_counters, splitk, vlogits, vkeys;
    float* splitk_ws = nullptr;
    size_t splitk_bytes = 0;
    bf16 *x = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *glog = nullptr, *grouped = nullptr,
         *act = nullptr, *y = nullptr, *tf16 = nullptr, *scratch_k = nullptr, *scratch_v = nullptr;
    float *rw = nullptr, *tf32 = nullptr, *partial = nullptr;
    int *ridx = nullptr, *perm = nullptr, *counts = nullptr, *cursor = nullptr, *offsets = nullptr, *tiles = nullptr,
        *recv_total = nullptr;
    size_t arena_bytes = 0;
    int launches = 0;

    void init(const Model& model, int batch, int rows_per_seq, int context, int mode, int win, bool selected_rows) {
        m = &model;
        B = batch;
        n = rows_per_seq;
        ctx = context;
        mask_mode = mode;
        window = win;
        int dev = 0;
        check(cudaGetDevice(&dev), "cudaGetDevice");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
        const Dims& d = model.dm;
        const size_t N = size_t(B) * n, P = N * d.k;
        rows = selected_rows ? B : int(N);
        key_chunk = 256;
        chunks = (ctx + n + key_chunk - 1) / key_chunk;
        const size_t heads = size_t(d.H + 2 * d.KV) * d.hd;
        // Expert parallel: the grouped expert inputs arrive in the group's receive buffer (up to cap rows from all
        // ranks); the expert activations and outputs cover those rows.
        const bool ep = model.ep != nullptr;
        if (ep && (long long)P > model.ep->pmax)
            throw ValueError("expert-parallel group sized for fewer (token, expert) pairs than this program routes");
        const size_t R = ep ? size_t(model.ep->cap) : P;
        // Flash decoding splits: about two CTAs per SM, whole 64-key tiles per split (at C5's 32 sequences x 8 KV heads
        // per GPU, 2 splits take 85 us per layer against 91 us for 4 and 98 us for 8: fewer, longer splits stream
        // better and merge less).
        // The TMA-staged decode kernel runs 4 CTAs per SM: at most that many CTAs, so one wave.
        if (ctx > 0) {
            const int tiles = (ctx + kFdKeys - 1) / kFdKeys;
            const int want = tma_attention() ? std::max(1, sms * 4 / (B * d.KV))
                                             : std::max(1, (sms * 2 + B * d.KV - 1) / (B * d.KV));
            fd_splits = std::min(tiles, want);
            fd_split_keys = (tiles + fd_splits - 1) / fd_splits * kFdKeys;
            fd_splits = (ctx + fd_split_keys - 1) / fd_split_keys;
        }
        std::vector<size_t> sizes = {
            N * d.d * 2, N * d.d * 2, N * heads * 2, N * d.H * d.hd * 2, N * d.H * d.hd * 2, N * d.E * 2,
            ep ? 0 : P * d.d * 2, R * d.I * 2, R * d.d * 2, size_t(rows) * d.d * 2, N * d.KV * d.hd * 2,
            N * d.KV * d.hd * 2, P * 4, size_t(rows) * d.d * 4, N * d.KV * d.G * size_t(chunks) * (d.hd + 2) * 4,
            P * 4, P * 4, size_t(d.E) * 4, size_t(d.E) * 4, size_t(d.E + 1) * 4, size_t(d.E + 1) * 4, 4,
            size_t(B) * d.KV * fd_splits * kFdRows * (2 + kFaDim) * 4,
        };
        std::vector<size_t> off(sizes.size());
        arena_bytes = 0;
        for (size_t i = 0; i < sizes.size(); ++i) {
            off[i] = arena_bytes;
            arena_bytes += (sizes[i] + 1023) / 1024 * 1024;
        }
        arena = DevBuf(arena_bytes);
        check(cudaMemset(arena.p, 0, arena_bytes), "arena");
        char* base = arena.as<char>();
        auto at = [&](int i) { return static_cast<void*>(base + off[size_t(i)]); };
        x = static_cast<bf16*>(at(0));
        xn = static_cast<bf16*>(at(1));
        qkv = static_cast<bf16*>(at(2));
        q = static_cast<bf16*>(at(3));
        attn = static_cast<bf16*>(at(4));
        glog = static_cast<bf16*>(at(5));
        grouped = static_cast<bf16*>(at(6));
        act = static_cast<bf16*>(at(7));
        y = static_cast<bf16*>(at(8));
        tf16 = static_cast<bf16*>(at(9));
        scratch_k = static_cast<bf16*>(at(10));
        scratch_v = static_cast<bf16*>(at(11));
        rw = static_cast<float*>(at(12));
        tf32 = static_cast<float*>(at(13));
        partial = static_cast<float*>(at(14));
        ridx = static_cast<int*>(at(15));
        perm = static_cast<int*>(at(16));
        counts = static_cast<int*>(at(17));
        cursor = static_cast<int*>(at(18));
        offsets = static_cast<int*>(at(19));
        tiles = static_cast<int*>(at(20));
        recv_total = static_cast<int*>(at(21));
        fd_part = static_cast<float*>(at(22));
        counters = DevBuf(N * d.KV * sizeof(unsigned));
        check(cudaMemset(counters.p, 0, counters.bytes), "attention counters");
        route_counters = DevBuf((N + kTileTokens - 1) / kTileTokens * sizeof(unsigned));
        check(cudaMemset(route_counters.p, 0, route_counters.bytes), "routing counters");
        // Split-K workspace for the dense projections of decode-sized row counts (QKV and out; the vocab GEMM has
        // enough tiles).
        for (const int cols : {int(heads), d.d}) {
            const int k = splitk_choice(int(N), cols, cols == d.d ? d.H * d.hd : d.d, 256, sms);
            if (k > 1) splitk_bytes = std::max(splitk_bytes, size_t(k) * N * size_t(cols) * 4);
        }
        if (splitk_bytes) {
            splitk = DevBuf(splitk_bytes);
            splitk_ws = splitk.as<float>();
        }
        if (model.ep && model.ep->vrows_max > 0) {  // vocab column shard
            if (rows > model.ep->vrows_max)
                throw ValueError("expert-parallel group's vocab shard sized for fewer final rows than this program selects");
            const size_t all = size_t(model.ep->world) * rows;
            vlogits = DevBuf(all * size_t(std::max(1, model.ep->vocab_rows_here())) * 2);
            vkeys = DevBuf(all * 8);
        }
    }

    // A (rows of another rank) is complete once each of `count` flags reaches *epoch.
    struct FlagWait {
        const unsigned* flags;
        int count;
        const unsigned* epoch;
        unsigned long long timeout_ns;
    };
    static FlagWait ep_wait(const EpArgs& a, const unsigned* flags) { return {flags, a.world, a.epoch, a.timeout_ns}; }

    // Outputs of the QKV GEMM's RoPE epilogue (kEpiRope): (cos, sin) table, new K and V rows, head counts.
    struct RopeOut {
        const float2* cs;
        bf16* k;
        bf16* v;
        int H, KV;
    };

    void gemm(cudaStream_t s, const bf16* A, int M, const bf16* W, int N, int K, int epi, const bf16* bias, bf16* C,
              int ldc, const bf16* residual, int groups, const int* offs, unsigned* err, const FlagWait* wait = nullptr,
              unsigned long long* argmax_keys = nullptr, int argmax_col_offset = 0, const RopeOut* rope = nullptr) {
        GemmArgs g{};
        if (rope) {
            g.rope_cs = rope->cs;
            g.rope_k = rope->k;
            g.rope_v = rope->v;
            g.rope_H = rope->H;
            g.rope_KV = rope->KV;
        }
        g.argmax_keys = argmax_keys;
        g.argmax_col_offset = argmax_col_offset;
        if (wait) {  // A arrives from the other ranks: wait for their flags in the prologue
            g.wait_flags = wait->flags;
            g.wait_count = wait->count;
            g.wait_epoch = wait->epoch;
            g.wait_timeout_ns = wait->timeout_ns;
        }
        g.M = M;
        g.N = N;
        g.K = K;
        g.epi = epi;
        g.bias = bias;
        g.residual = residual;
        g.ldr = N;
        g.C = C;
        g.ldc = ldc;
        g.alpha = m->dm.alpha;
        g.limit = m->dm.limit;
        g.groups = groups;
        g.offsets = offs;
        gemm_bf16(s, A, W, g, M, groups * N, tiles, sms, err, splitk_ws, splitk_bytes);
        launches += offs == nullptr && epi != kEpiRope && splitk_choice(M, N, K, N <= 32 ? 32 : 256, sms) > 1 ? 2 : 1;
    }

    void enqueue(cudaStream_t s, const GptIO& io, unsigned* err) {
        const Dims& dm = m->dm;
        const int N = B * n, P = N * dm.k, L = m->desc.layers;
        const int heads = (dm.H + 2 * dm.KV) * dm.hd;
        launches = 0;
        launch(s, dim3(N), dim3(128), 0, k_embed_bf16, io.tokens, N, reinterpret_cast<const bf16*>(m->at(0)), dm.V, dm.d,
               x, err);
        ++launches;
        // CHROMA_B200_NO_FLASH selects the split-KV SIMT attention for every chunk (a cross-check of the two kernels).
        static const bool no_flash = std::getenv("CHROMA_B200_NO_FLASH") != nullptr;
        const bool flash = !no_flash && n >= 16 && mask_mode != kMaskBuffer && ctx <= kFaMaxCacheTiles * kFaKeys;
        // RoPE in the QKV GEMM's epilogue (no k_rope_split launch, no re-read of the QKV output) where that GEMM runs
        // without split-K; the (cos, sin) table of this forward's positions then lives in the unused QKV buffer.
        // CHROMA_B200_ROPE_EPILOGUE=0 keeps the separate kernel.
        static const char* rope_env = std::getenv("CHROMA_B200_ROPE_EPILOGUE");
        const bool rope_fused = !(rope_env && rope_env[0] == '0') && dm.hd == 64 &&
                                splitk_choice(N, heads, dm.d, 256, sms) == 1;
        const float2* rope_cs = reinterpret_cast<const float2*>(qkv);
        if (rope_fused) {
            launch(s, dim3(unsigned((N * (dm.hd / 2) + 255) / 256)), dim3(256), 0, k_rope_table, io.positions,
                   m->inv_freq.as<const float>(), dm.conc, N, dm.hd / 2, reinterpret_cast<float2*>(qkv));
            ++launches;
        }
        for (int l = 0; l < L; ++l) {
            const LayerW<bf16> w = m->layer<bf16>(l);
            bf16* nk;
            bf16* nv;
            const bf16* ck;
            const bf16* cv;
            if (m->desc.kind == CHROMA_B200_GPTOSS_CACHED) {
                nk = static_cast<bf16*>(io.new_k) + size_t(l) * N * dm.KV * dm.hd;
                nv = static_cast<bf16*>(io.new_v) + size_t(l) * N * dm.KV * dm.hd;
                ck = static_cast<const bf16*>(io.cache_k) + size_t(l) * ctx * dm.KV * dm.hd;
                cv = static_cast<const bf16*>(io.cache_v) + size_t(l) * ctx * dm.KV * dm.hd;
            } else {
                nk = scratch_k;
                nv = scratch_v;
                ck = nk;
                cv = nv;
            }
            if (l == 0) {  // later layers: the previous layer's combine already wrote this norm
                launch(s, dim3(N), dim3(256), 0, k_rms_bf16, x, dm.d, dm.eps, w.attn_norm, xn);
                ++launches;
            }
            if (rope_fused) {
                const RopeOut ro{rope_cs, nk, nv, dm.H, dm.KV};
                gemm(s, xn, N, w.qkv_w, heads, dm.d, kEpiRope, w.qkv_b, q, dm.H * dm.hd, nullptr, 1, nullptr, err,
                     nullptr, nullptr, 0, &ro);
            } else {
                gemm(s, xn, N, w.qkv_w, heads, dm.d, kEpiStore, w.qkv_b, qkv, heads, nullptr, 1, nullptr, err);
                launch(s, dim3(N), dim3(256), 0, k_rope_split, qkv, dm.H, dm.KV, dm.hd, io.positions,
                       m->inv_freq.as<const float>(), dm.conc, q, nk, nv);
            }
            const bool windowed = m->layer_window[size_t(l)] != 0;
            const int win = mask_mode == kMaskSlots ? (windowed ? window : ctx) : (windowed ? window : 0);
            if (flash) {
                FlashArgs fa;
                fa.n = n;
                fa.ctx = ctx;
                fa.B = B;
                fa.H = dm.H;
                fa.KV = dm.KV;
                fa.G = dm.G;
                fa.cache_seq_stride = size_t(L) * ctx * dm.KV * dm.hd;
                fa.window = win;
                fa.scale_log2 = dm.sm_scale * 1.4426950408889634f;
                fa.slots = mask_mode == kMaskSlots ? io.slots : nullptr;
                fa.pos0 = mask_mode == kMaskSlots ? io.pos0 : nullptr;
                if (mask_mode != kMaskSlots) fa.ctx = 0;
                if (tma_attention()) {
                    // tcgen05 flash attention: Q, K, V tiles through TMA tensor maps.
                    FlashMaps fm;
                    const uint64_t KVb = uint64_t(dm.KV) * 128;
                    {
                        const uint64_t dims[3] = {64, uint64_t(dm.H), uint64_t(N)};
                        const uint64_t st[2] = {128, uint64_t(dm.H) * 128};
                        const uint32_t box[3] = {64, 1, kFtRows};
                        fm.q = bf16_map_nd(q, 3, dims, st, box);
                    }
                    {
                        const uint64_t dims[3] = {64, uint64_t(dm.KV), uint64_t(N)};
                        const uint64_t st[2] = {128, KVb};
                        const uint32_t box[3] = {64, 1, kFtKeys};
                        fm.kn = bf16_map_nd(nk, 3, dims, st, box);
                        fm.vn = bf16_map_nd(nv, 3, dims, st, box);
                    }
                    if (fa.ctx > 0) {
                        const uint64_t dims[4] = {64, uint64_t(dm.KV), uint64_t(ctx), uint64_t(B)};
                        const uint64_t st[3] = {128, KVb, uint64_t(L) * ctx * KVb};
                        const uint32_t box[4] = {64, 1, kFtKeys, 1};
                        fm.kc = bf16_map_nd(ck, 4, dims, st, box);
                        fm.vc = bf16_map_nd(cv, 4, dims, st, box);
                    } else {
                        fm.kc = fm.kn;
                        fm.vc = fm.vn;
                    }
                    launch(s, dim3((n + kFtQ * kFtRows - 1) / (kFtQ * kFtRows), dm.H, B), dim3(kFtThreads), kFtSmemBytes,
                           k_flash_prefill_tc, fm, fa, w.sinks, attn, err);
                } else
                launch(s, dim3((n + kFaRows - 1) / kFaRows, dm.H, B), dim3(kFaThreads), kFaSmemBytes, k_flash_prefill, q, fa, ck, cv,
                       static_cast<const bf16*>(nk), static_cast<const bf16*>(nv), w.sinks, attn);
            } else if (mask_mode == kMaskSlots && n * dm.G <= kFdRows) {
                DecodeArgs a;
                a.n = n;
                a.ctx = ctx;
                a.B = B;
                a.H = dm.H;
                a.KV = dm.KV;
                a.G = dm.G;
                a.splits = fd_splits;
                a.split_keys = fd_split_keys;
                a.cache_seq_stride = size_t(L) * ctx * dm.KV * dm.hd;
                a.window = win;
                a.scale_log2 = dm.sm_scale * 1.4426950408889634f;
                a.slots = io.slots;
                a.pos0 = io.pos0;
                a.part = fd_part;
                a.counters = counters.as<unsigned>();
                if (tma_attention()) {
                    FlashMaps fm;
                    const uint64_t KVb = uint64_t(dm.KV) * 128;
                    {
                        const uint64_t dims[3] = {64, uint64_t(dm.KV), uint64_t(N)};
                        const uint64_t st[2] = {128, KVb};
                        const uint32_t box[3] = {64, 1, kFdKeys};
                        fm.kn = bf16_map_nd(nk, 3, dims, st, box);
                        fm.vn = bf16_map_nd(nv, 3, dims, st, box);
                    }
                    {
                        const uint64_t dims[4] = {64, uint64_t(dm.KV), uint64_t(ctx), uint64_t(B)};
                        const uint64_t st[3] = {128, KVb, uint64_t(L) * ctx * KVb};
                        const uint32_t box[4] = {64, 1, kFdKeys, 1};
                        fm.kc = bf16_map_nd(ck, 4, dims, st, box);
                        fm.vc = bf16_map_nd(cv, 4, dims, st, box);
                    }
                    fm.q = fm.kn;  // unused
                    launch(s, dim3(B, dm.KV, fd_splits), dim3(kFdtThreads), kFdtSmemBytes, k_flash_decode_tma, fm, q, a,
                           w.sinks, attn, err);
                } else
                launch(s, dim3(B, dm.KV, fd_splits), dim3(kFdThreads), kFdSmemBytes, k_flash_decode, q, a, ck, cv,
                       static_cast<const bf16*>(nk), static_cast<const bf16*>(nv), w.sinks, attn);
            } else {
                AttnArgs a;
                a.n = n;
                a.ctx = ctx;
                a.B = B;
                a.chunks = chunks;
                a.key_chunk = key_chunk;
                a.cache_seq_stride = size_t(L) * ctx * dm.KV * dm.hd;
                a.mask_mode = mask_mode;
                a.window = win;
                a.slots = io.slots;
                a.pos0 = io.pos0;
                a.partial = partial;
                a.counters = counters.as<unsigned>();
                const bf16* bias = static_cast<const bf16*>(windowed ? io.window_mask : io.mask);
                const size_t smem = (size_t(2) * key_chunk * (dm.hd + 1) + size_t(dm.G) * key_chunk + size_t(dm.G) * dm.hd) * 4;
                launch(s, dim3(n, dm.KV, B * chunks), dim3(kThreads), smem, k_attention<bf16, bf16>, q, dm, a, ck, cv,
                       static_cast<const bf16*>(nk), static_cast<const bf16*>(nv), bias, w.sinks, attn);
            }
            gemm(s, attn, N, w.out_w, dm.d, dm.H * dm.hd, kEpiResidual, w.out_b, x, dm.d, x, 1, nullptr, err);
            {
                int* rec = io.routes ? io.routes + size_t(l) * N * dm.k : static_cast<int*>(nullptr);
                const int tiles_t = (N + kTileTokens - 1) / kTileTokens;
                if (tiles_t >= sms) {
                    // Many tokens: norm, gate logits on the tensor cores, then top-k + counts.
                    launch(s, dim3(N), dim3(256), 0, k_rms_bf16, x, dm.d, dm.eps, w.mlp_norm, xn);
                    gemm(s, xn, N, w.gate_w, dm.E, dm.d, kEpiStore, w.gate_b, glog, dm.E, nullptr, 1, nullptr, err);
                    launch(s, dim3(unsigned((N + 7) / 8)), dim3(256), 0, k_route_topk, static_cast<const bf16*>(glog), N,
                           dm.E, dm.k, ridx, rw, rec, counts);
                    ++launches;
                } else {
                    // Decode-sized: one fused kernel; experts split over CTAs so the gate weights stream from ~1 wave.
                    const int epc = std::max(8, (dm.E * tiles_t + sms - 1) / sms);
                    const unsigned eb = unsigned((dm.E + epc - 1) / epc);
                    const size_t smem = (size_t(kTileTokens) * (dm.d + dm.E) + kTileTokens) * 4;
                    launch(s, dim3(unsigned(tiles_t), eb), dim3(kThreads), smem, k_route_fused,
                           static_cast<const bf16*>(x), N, dm.d, dm.eps, w.mlp_norm, w.gate_w, w.gate_b, dm.E, epc, dm.k,
                           xn, glog, ridx, rw, rec, counts, route_counters.as<unsigned>());
                }
            }
            CombineExtra ex{};
            if (l + 1 < L) {  // fuse the next layer's attention norm into the combine
                ex.norm_w = m->layer<bf16>(l + 1).attn_norm;
                ex.eps = dm.eps;
                ex.xn = xn;
            }
            if (m->ep) {
                enqueue_ep_experts(s, w, ex, err);
            } else {
                launch(s, dim3(1), dim3(32), 0, k_route_offsets, counts, dm.E, offsets, cursor);
                launch(s, dim3((P + 7) / 8), dim3(256), 0, k_route_scatter, ridx, P, dm.k, dm.d, xn, cursor, perm,
                       grouped);
                gemm(s, grouped, P, w.w1, 2 * dm.I, dm.d, kEpiSwiglu, w.b1, act, dm.I, nullptr, dm.E, offsets, err);
                gemm(s, act, P, w.w2, dm.d, dm.I, kEpiExpert, w.b2, y, dm.d, nullptr, dm.E, offsets, err);
                launch(s, dim3(N), dim3(256), 0, k_moe_combine, static_cast<const bf16*>(y), static_cast<const int*>(perm),
                       static_cast<const float*>(rw), dm.k, dm.d, x, ex);
                launches += 3;
            }
            launches += rope_fused ? 2 : 3;
        }
        launch(s, dim3(rows), dim3(256), 0, k_norm_rows, x, rows, io.rows, n, reinterpret_cast<const float*>(m->at(1)),
               dm.d, dm.eps, tf32, tf16, io.keys, err);
        ++launches;
        enqueue_vocab(s, io, err);
    }

    // The experts of one layer across the expert-parallel group (ep.cuh): counts to every rank, row plan, dispatch
    // of the (token, slot) rows to their owners, grouped GEMMs over the rows this rank received, return of the
    // outputs to their sources, weighted combine in slot order.
    void enqueue_ep_experts(cudaStream_t s, const LayerW<bf16>& w, CombineExtra ex, unsigned* err) {
        const Dims& dm = m->dm;
        const EpGroup& g = *m->ep;
        const EpArgs a = g.args(m->El);
        const int N = B * n, P = N * dm.k, cap = int(g.cap);
        launch(s, dim3(1), dim3(256), 0, k_ep_counts, a, counts, cursor, offsets, recv_total, err);
        launch(s, dim3(unsigned(std::max(1, std::min((P + 7) / 8, sms * 4)))), dim3(256), 0, k_ep_dispatch, a,
               static_cast<const int*>(ridx), P, dm.k, static_cast<const bf16*>(xn), cursor, err);
        const FlagWait dispatched = ep_wait(a, &reinterpret_cast<const EpHeader*>(a.peer[a.rank])->disp_flag[0]);
        gemm(s, g.recv_rows(), cap, w.w1, 2 * dm.I, dm.d, kEpiSwiglu, w.b1, act, dm.I, nullptr, m->El, offsets, err,
             &dispatched);
        gemm(s, act, cap, w.w2, dm.d, dm.I, kEpiExpert, w.b2, y, dm.d, nullptr, m->El, offsets, err);
        launch(s, dim3(unsigned(std::max(1, std::min(sms * 4, (cap + 7) / 8)))), dim3(256), 0, k_ep_return, a,
               static_cast<const bf16*>(y),
               static_cast<const int*>(recv_total), err);
        ex.wait_flags = &reinterpret_cast<const EpHeader*>(a.peer[a.rank])->comb_flag[0];
        ex.wait_count = a.world;
        ex.wait_epoch = a.epoch;
        ex.wait_timeout_ns = a.timeout_ns;
        ex.err = err;
        launch(s, dim3(N), dim3(256), 0, k_moe_combine, static_cast<const bf16*>(g.return_rows()),
               static_cast<const int*>(nullptr), static_cast<const float*>(rw), dm.k, dm.d, x, ex);
        launches += 4;
    }

    void enqueue_vocab(cudaStream_t s, const GptIO& io, unsigned* err) {
        const Dims& dm = m->dm;
        const bf16* W = reinterpret_cast<const bf16*>(m->at(2));
        if (m->ep && m->ep->vrows_max > 0) {
            // Vocab column shard (ep.cuh): all ranks' final rows x this rank's vocab rows; keys/logits to the owners.
            const EpGroup& g = *m->ep;
            const EpArgs a = g.args(m->El);
            const int Vr = g.vocab_rows_here(), all = g.world * rows;
            const bool want_logits = io.keys == nullptr;
            launch(s, dim3(unsigned(std::max(1, std::min(sms, (all + 7) / 8)))), dim3(256), 0, k_vocab_share_rows, a,
                   static_cast<const bf16*>(tf16), rows, vkeys.as<unsigned long long>());
            const FlagWait gathered = ep_wait(a, &reinterpret_cast<const EpHeader*>(a.peer[a.rank])->vrow_flag[0]);
            gemm(s, reinterpret_cast<const bf16*>(a.peer[a.rank] + a.off_vrows), all, W, Vr, dm.d, kEpiStore, nullptr,
                 vlogits.as<bf16>(), Vr, nullptr, 1, nullptr, err, &gathered, vkeys.as<unsigned long long>(),
                 g.rank * g.Vl);
            launch(s, dim3(unsigned(std::max(1, std::min(sms, (all + 7) / 8)))), dim3(256), 0, k_vocab_return, a,
                   static_cast<const unsigned long long*>(vkeys.as<unsigned long long>()),
                   static_cast<const bf16*>(vlogits.as<bf16>()), Vr, rows, int(want_logits));
            launch(s, dim3(unsigned(want_logits ? sms : 1)), dim3(256), 0, k_vocab_finish, a, rows, io.keys,
                   static_cast<bf16*>(io.logits), int(want_logits), err);
            launches += 3;
            return;
        }
        if (rows < 16) {
            launch_vocab<bf16>(s, dm, sms, tf32, rows, W, static_cast<bf16*>(io.logits), io.keys, err);
            ++launches;
        } else {  // greedy argmax fused into the GEMM epilogue (keys zeroed by k_norm_rows)
            gemm(s, tf16, rows, W, dm.V, dm.d, kEpiStore, nullptr, static_cast<bf16*>(io.logits), dm.V, nullptr, 1, nullptr,
                 err, nullptr, io.keys);
        }
    }
};

struct GptExec {
    const Model* m = nullptr;
    int B = 1, n = 1, ctx = 0, mask_mode = kMaskBuffer, window = 0, sms = 148, chunks = 1, key_chunk = 256;
    DevBuf arena, counters;
    size_t arena_bytes = 0, unreused_bytes = 0;
    float *x = nullptr, *x2 = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *rw = nullptr, *tf = nullptr,
          *partial = nullptr;
    int* ridx = nullptr;
    void *scratch_k = nullptr, *scratch_v = nullptr;
    GptIO io;
    unsigned* err = nullptr;
    int launches = 0;

    // Temporaries with their kernel-index lifetimes (0 embedding; per layer l: 1+5l QKV, 2+5l attention, 3+5l out,
    // 4+5l router + expert up, 5+5l expert down; 1+5L final norm; 2+5L vocab), in planning order.
    bool large_path = false;
    LargeExec large;

    // Layer-weight prefetch (dev-sized models): every layer's weights (a contiguous range of the weights buffer,
    // ~30 MB for the dev model) are pulled into L2 by a kernel on a side stream at the start of each step, so the
    // latency-bound layer kernels, the MoE ones whose weights depend on the routing included, hit L2.
    cudaStream_t side = nullptr;
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    const char* prefetch_base = nullptr;
    size_t prefetch_bytes = 0;

    // One-token decode of dev-sized fp32 models: every layer in one cluster launch (decode_cluster.cuh).
    bool cluster_decode = false;
    int dc_kpc = 0;
    size_t dc_smem = 0;
    void (*dc_kernel)(DecodeClusterArgs) = nullptr;
    // Forward of up to 8 tokens of dev-sized fp32 uncached programs: every layer in one cluster launch
    // (fwd_cluster.cuh).
    bool cluster_fwd = false;
    size_t fc_smem = 0;
    // Expert-grouped MoE for 16+ tokens of d = I = 128 programs (gptoss.cuh k_route_rows ... k_moe_combine_rows;
    // CHROMA_B200_PER_SLOT_MOE keeps k_moe_up / k_moe_down, whose results are the same bits).
    bool grouped_moe = false;
    DevBuf g_xn, g_lists, g_counts, g_ys;
    bool skip_vocab = false;  // set while enqueue_layers runs the per-layer chain
    DevBuf dc_layers, dc_windows;

    GptExec() = default;
    GptExec(const GptExec&) = delete;
    GptExec& operator=(const GptExec&) = delete;
    ~GptExec() {
        if (side) cudaStreamDestroy(side);
        if (fork_ev) cudaEventDestroy(fork_ev);
        if (join_ev) cudaEventDestroy(join_ev);
    }

    void init(const Model& model, int batch, int rows_per_seq, int context, int mode, int win, bool selected_rows) {
        m = &model;
        B = batch;
        n = rows_per_seq;
        ctx = context;
        mask_mode = mode;
        window = win;
        if (is_large(model.desc)) {
            large_path = true;
            large.init(model, batch, rows_per_seq, context, mode, win, selected_rows);
            arena_bytes = unreused_bytes = large.arena_bytes;
            return;
        }
        int dev = 0;
        check(cudaGetDevice(&dev), "cudaGetDevice");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
        const Dims& d = model.dm;
        const int L = model.desc.layers;
        const size_t N = size_t(B) * n;
        const int last = 5 * (L - 1);
        {
            const size_t first = size_t(model.offsets.at(3));
            const size_t bytes = size_t(model.desc.weight_bytes) - first;
            if (bytes <= (size_t(48) << 20)) {
                prefetch_base = model.weights->ptr + first;
                prefetch_bytes = bytes;
                check(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "prefetch stream");
                check(cudaEventCreateWithFlags(&fork_ev, cudaEventDisableTiming), "prefetch event");
                check(cudaEventCreateWithFlags(&join_ev, cudaEventDisableTiming), "prefetch event");
            }
        }
        key_chunk = d.hd <= 32 ? 512 : 256;
        // fp32 programs split the keys into 64-key chunks merged by the last CTA, so decode batches fill the GPU
        // (batch 64: 320 CTAs instead of 64 whole-ring ones). bf16 programs keep whole chunks: a single chunk
        // rounds the probabilities where the reference does.
        if (model.desc.storage == CHROMA_B200_FP32) key_chunk = 64;
        chunks = (ctx + n + key_chunk - 1) / key_chunk;
        auto round = [](size_t b) { return (b + 255) / 256 * 256; };
        std::vector<Alloc> a = {
            {round(N * d.d * 4), 0, 1 + 5 * L, 0},                                  // x
            {round(N * d.H * d.hd * 4), 1, 2 + last, 0},                             // q
            {round(N * d.H * d.hd * 4), 2, 3 + last, 0},                             // attn
            {round(N * d.d * 4), 3, 5 + last, 0},                                    // x2
            {round(N * d.k * 4), 4, 5 + last, 0},                                    // ridx
            {round(N * d.k * 4), 4, 5 + last, 0},                                    // rw
            {round(N * d.k * d.I * 4), 4, 5 + last, 0},                              // act
            {round(N * d.KV * d.G * size_t(chunks) * (d.hd + 2) * 4), 2, 2 + last, 0},  // partial
            {round(N * d.d * 4), 1 + 5 * L, 2 + 5 * L, 0},                          // tf
        };
        const bool uncached = model.desc.kind != CHROMA_B200_GPTOSS_CACHED;
        if (uncached) {
            const size_t es = storage_size(model.desc.storage);
            a.push_back({round(N * d.KV * d.hd * es), 1, 2 + last, 0});  // scratch_k
            a.push_back({round(N * d.KV * d.hd * es), 1, 2 + last, 0});  // scratch_v
        }
        unreused_bytes = 0;
        for (const auto& x_ : a) unreused_bytes += x_.size;
        arena_bytes = plan_arena(a);
        arena = DevBuf(arena_bytes);
        char* base = arena.as<char>();
        x = reinterpret_cast<float*>(base + a[0].offset);
        q = reinterpret_cast<float*>(base + a[1].offset);
        attn = reinterpret_cast<float*>(base + a[2].offset);
        x2 = reinterpret_cast<float*>(base + a[3].offset);
        ridx = reinterpret_cast<int*>(base + a[4].offset);
        rw = reinterpret_cast<float*>(base + a[5].offset);
        act = reinterpret_cast<float*>(base + a[6].offset);
        partial = reinterpret_cast<float*>(base + a[7].offset);
        tf = reinterpret_cast<float*>(base + a[8].offset);
        if (uncached) {
            scratch_k = base + a[9].offset;
            scratch_v = base + a[10].offset;
        }
        counters = DevBuf(N * d.KV * sizeof(unsigned));
        check(cudaMemset(counters.p, 0, counters.bytes), "attention counters");
        if (N >= 16 && d.d == 128 && d.I == 128 && std::getenv("CHROMA_B200_PER_SLOT_MOE") == nullptr) {
            grouped_moe = true;
            g_xn = DevBuf(N * d.d * 4);
            g_lists = DevBuf(size_t(d.E) * N * 4);
            g_counts = DevBuf(size_t(d.E) * 4);
            check(cudaMemset(g_counts.p, 0, g_counts.bytes), "expert counts");
            g_ys = DevBuf(N * d.k * d.d * 4);
        }
        init_cluster_decode();
        init_cluster_fwd();
    }

    // The forward cluster takes the uncached fp32 programs of up to 8 tokens at batch 1 whose widths fit its fixed
    // work split (d = H*hd = I = 128, head_dim 16, QKV rows <= 2 per warp, one warp per (row, head), k <= 4,
    // E <= 16) and whose layers are packed layer-major. CHROMA_B200_FWD_CLUSTER=0 keeps the per-layer kernels.
    void init_cluster_fwd() {
        const Dims& d = m->dm;
        const int L = m->desc.layers;
        const char* env = std::getenv("CHROMA_B200_FWD_CLUSTER");
        if (env && env[0] == '0') return;
        if (m->desc.storage != CHROMA_B200_FP32) return;
        if (m->desc.kind != CHROMA_B200_GPTOSS_FORWARD && m->desc.kind != CHROMA_B200_GPTOSS_LAST) return;
        if (mask_mode != kMaskCausal || ctx != 0 || B != 1 || n < 1 || n > kFcTok) return;
        if (d.d != 128 || d.H * d.hd != 128 || d.I != 128 || d.hd != 16) return;
        if ((d.H + 2 * d.KV) * d.hd > kDcRows1 * kDcWarps || n * d.H > kDcWarps) return;
        if ((d.H + 2 * d.KV) * d.hd % 8 != 0) return;  // each CTA's 8-row QKV blocks are whole
        if (d.k > kDcMaxK || d.E > kDcMaxE || d.E < d.k) return;
        if (reinterpret_cast<uintptr_t>(m->weights->ptr) % 16 != 0) return;  // bulk L2 prefetch of each layer
        for (int l = 0; l + 1 < L; ++l)
            if (m->offsets.at(size_t(3 + 13 * (l + 1))) < m->offsets.at(size_t(3 + 13 * l))) return;
        const FcLayout lay(d, L);
        const size_t smem = size_t(lay.total) * 4;
        if (smem + 1024 > 227 * 1024) return;
        ClusterLaunch cl(nullptr, dim3(kDcC), dim3(kThreads), smem, kDcC, k_fwd_cluster<16>);
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, k_fwd_cluster<16>, &cl.cfg) != cudaSuccess || clusters < 1) {
            cudaGetLastError();
            return;
        }
        std::vector<LayerW<float>> lw(static_cast<size_t>(L));
        std::vector<int> win(static_cast<size_t>(L));
        for (int l = 0; l < L; ++l) {
            lw[size_t(l)] = m->layer<float>(l);
            win[size_t(l)] = m->layer_window[size_t(l)] != 0 ? window : 0;
        }
        dc_layers = DevBuf(lw.size() * sizeof(LayerW<float>));
        dc_windows = DevBuf(win.size() * sizeof(int));
        check(cudaMemcpy(dc_layers.p, lw.data(), dc_layers.bytes, cudaMemcpyHostToDevice), "cluster layer table");
        check(cudaMemcpy(dc_windows.p, win.data(), dc_windows.bytes, cudaMemcpyHostToDevice), "cluster window table");
        fc_smem = smem;
        cluster_fwd = true;
        // Beside the (L2-prefetching) cluster kernel, the side stream pulls the vocab matrix into L2.
        if (!side) {
            check(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "prefetch stream");
            check(cudaEventCreateWithFlags(&fork_ev, cudaEventDisableTiming), "prefetch event");
            check(cudaEventCreateWithFlags(&join_ev, cudaEventDisableTiming), "prefetch event");
        }
        prefetch_base = m->at(2);
        prefetch_bytes = (size_t(d.V) * d.d * 4) & ~size_t(15);
    }

    void enqueue_cluster_fwd(cudaStream_t s) {
        FwdClusterArgs a;
        a.dm = m->dm;
        a.L = m->desc.layers;
        a.n = n;
        a.layers = dc_layers.as<const LayerW<float>>();
        a.windows = dc_windows.as<const int>();
        a.emb = reinterpret_cast<const float*>(m->at(0));
        a.final_norm = reinterpret_cast<const float*>(m->at(1));
        a.inv_freq = m->inv_freq.as<const float>();
        a.positions = io.positions;
        a.tokens = io.tokens;
        a.rows = io.rows;
        a.routes = io.routes;
        a.tf = tf;
        a.keys = io.keys;
        a.err = err;
        ClusterLaunch cl(s, dim3(kDcC), dim3(kThreads), fc_smem, kDcC, k_fwd_cluster<16>);
        check(cudaLaunchKernelEx(&cl.cfg, k_fwd_cluster<16>, a), "cluster forward launch");
    }

    // The cluster path takes a single new token of a cached fp32 program whose widths fit its fixed work split
    // (d = H*hd = I = 128: one row of 128 per warp and lane-float4, one mlp1 pair and one mlp2 row of each expert
    // per warp; QKV rows <= 2 per warp; k <= 4; E <= 16 gate rows; head_dim 16; ctx + 1 keys over 16 CTAs of at
    // most 32 keys) and whose shared memory fits. CHROMA_B200_DECODE_CLUSTER=0 keeps the per-layer kernels.
    void init_cluster_decode() {
        const Dims& d = m->dm;
        const int L = m->desc.layers;
        const char* env = std::getenv("CHROMA_B200_DECODE_CLUSTER");
        if (env && env[0] == '0') return;
        if (m->desc.storage != CHROMA_B200_FP32 || m->desc.kind != CHROMA_B200_GPTOSS_CACHED) return;
        if (mask_mode != kMaskSlots || B * n != 1) return;
        if (d.d != 128 || d.H * d.hd != 128 || d.I != 128) return;
        if ((d.H + 2 * d.KV) * d.hd > kDcRows1 * kDcWarps || d.k > kDcMaxK) return;
        if (reinterpret_cast<uintptr_t>(m->weights->ptr) % 16 != 0) return;  // bulk L2 prefetch of each layer
        if (d.E > kDcMaxE || d.E < d.k || d.hd != 16) return;
        const int kpc = (ctx + 1 + kDcC - 1) / kDcC;
        if (kpc > 32) return;
        const DcLayout lay(d, L, kpc);
        const size_t smem = size_t(lay.total) * 4;
        if (smem + 1024 > 227 * 1024) return;
        dc_kernel = k_decode_cluster<1, 16>;
        ClusterLaunch cl(nullptr, dim3(kDcC), dim3(kThreads), smem, kDcC, dc_kernel);
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, dc_kernel, &cl.cfg) != cudaSuccess || clusters < 1) {
            cudaGetLastError();
            return;
        }
        std::vector<LayerW<float>> lw(static_cast<size_t>(L));
        std::vector<int> win(static_cast<size_t>(L));
        for (int l = 0; l < L; ++l) {
            lw[size_t(l)] = m->layer<float>(l);
            win[size_t(l)] = m->layer_window[size_t(l)] != 0 ? window : ctx;
        }
        dc_layers = DevBuf(lw.size() * sizeof(LayerW<float>));
        dc_windows = DevBuf(win.size() * sizeof(int));
        check(cudaMemcpy(dc_layers.p, lw.data(), dc_layers.bytes, cudaMemcpyHostToDevice), "cluster layer table");
        check(cudaMemcpy(dc_windows.p, win.data(), dc_windows.bytes, cudaMemcpyHostToDevice), "cluster window table");
        for (int l = 0; l + 1 < L; ++l)  // the per-layer L2 prefetch relies on each layer's tensors being contiguous
            if (m->offsets.at(size_t(3 + 13 * (l + 1))) < m->offsets.at(size_t(3 + 13 * l))) return;
        dc_kpc = kpc;
        dc_smem = smem;
        cluster_decode = true;
        // Beside the (L2-prefetching) cluster kernel, the side stream pulls the vocab matrix into L2 for the vocab GEMV.
        if (!side) {
            check(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking), "prefetch stream");
            check(cudaEventCreateWithFlags(&fork_ev, cudaEventDisableTiming), "prefetch event");
            check(cudaEventCreateWithFlags(&join_ev, cudaEventDisableTiming), "prefetch event");
        }
        prefetch_base = m->at(2);
        prefetch_bytes = (size_t(d.V) * d.d * 4) & ~size_t(15);
    }

    // Kernels of this repository one enqueue() launches (the side-stream prefetch included).
    int planned_launches() const {
        if (large_path) return large.launches;
        const int pre = side ? 1 : 0;
        const bool fused_or = grouped_moe && m->dm.H * m->dm.hd == 128 && m->dm.E <= 2 * kWarps;
        return (cluster_decode || cluster_fwd) ? pre + 2
                                               : pre + 1 + (grouped_moe ? (fused_or ? 6 : 7) : 5) * m->desc.layers + 2;
    }

    void enqueue_cluster_decode(cudaStream_t s) {
        DecodeClusterArgs a;
        a.dm = m->dm;
        a.L = m->desc.layers;
        a.ctx = ctx;
        a.kpc = dc_kpc;
        a.layers = dc_layers.as<const LayerW<float>>();
        a.windows = dc_windows.as<const int>();
        a.emb = reinterpret_cast<const float*>(m->at(0));
        a.final_norm = reinterpret_cast<const float*>(m->at(1));
        a.inv_freq = m->inv_freq.as<const float>();
        a.tokens = io.tokens;
        a.pos0 = io.pos0;
        a.slots = io.slots;
        a.cache_k = static_cast<const float*>(io.cache_k);
        a.cache_v = static_cast<const float*>(io.cache_v);
        a.new_k = static_cast<float*>(io.new_k);
        a.new_v = static_cast<float*>(io.new_v);
        a.routes = io.routes;
        a.rows = io.commit_k ? nullptr : io.rows;  // device-resident steps always take their single new row
        a.tf = tf;
        a.keys = io.keys;
        a.err = err;
        a.commit_k = static_cast<float*>(io.commit_k);
        a.commit_v = static_cast<float*>(io.commit_v);
        a.commit_slots = io.commit_slots;
        ClusterLaunch cl(s, dim3(kDcC), dim3(kThreads), dc_smem, kDcC, dc_kernel);
        check(cudaLaunchKernelEx(&cl.cfg, dc_kernel, a), "cluster decode launch");
    }

    template <typename T> void enqueue_t(cudaStream_t s) {
        const Dims& dm = m->dm;
        const int N = B * n;
        const int L = m->desc.layers;
        launches = 0;
        if (side) {  // fork: the prefetch runs beside the whole step and joins at its end
            check(cudaEventRecord(fork_ev, s), "prefetch fork");
            check(cudaStreamWaitEvent(side, fork_ev, 0), "prefetch fork");
            if (cluster_decode || cluster_fwd) k_prefetch_l2_bulk<<<8, 256, 0, side>>>(prefetch_base, prefetch_bytes);
            else k_prefetch_l2<<<64, 256, 0, side>>>(prefetch_base, prefetch_bytes);
            check(cudaGetLastError(), "prefetch launch");
            check(cudaEventRecord(join_ev, side), "prefetch join");
            ++launches;
        }
        if constexpr (std::is_same_v<T, float>) {
            if (cluster_decode || cluster_fwd) {
                if (cluster_decode) enqueue_cluster_decode(s);
                else enqueue_cluster_fwd(s);
                enqueue_vocab_t<T>(s);
                launches += 2;
                if (side) check(cudaStreamWaitEvent(s, join_ev, 0), "prefetch join");
                return;
            }
        }
        launch(s, dim3(N), dim3(128), 0, k_embed<T>, io.tokens, N, reinterpret_cast<const T*>(m->at(0)), dm.V, dm.d, x,
               err);
        ++launches;
        const int heads_total = dm.H + 2 * dm.KV;
        const int tiles = (N + kTileTokens - 1) / kTileTokens;
        const size_t smem_in = size_t(kTileTokens) * (dm.d + dm.hd + 1) * 4;
        const size_t smem_attn = (size_t(2) * key_chunk * (dm.hd + 1) + size_t(dm.G) * key_chunk + size_t(dm.G) * dm.hd) * 4;
        const size_t smem_out = size_t(kTileTokens) * dm.H * dm.hd * 4;
        const size_t smem_up = size_t(dm.d + dm.E + 17) * 4;
        for (int l = 0; l < L; ++l) {
            const LayerW<T> w = m->layer<T>(l);
            T* nk;
            T* nv;
            const T* ck = nullptr;
            const T* cv = nullptr;
            if (m->desc.kind == CHROMA_B200_GPTOSS_CACHED) {
                nk = static_cast<T*>(io.new_k) + size_t(l) * N * dm.KV * dm.hd;
                nv = static_cast<T*>(io.new_v) + size_t(l) * N * dm.KV * dm.hd;
                ck = static_cast<const T*>(io.cache_k) + size_t(l) * ctx * dm.KV * dm.hd;
                cv = static_cast<const T*>(io.cache_v) + size_t(l) * ctx * dm.KV * dm.hd;
            } else {
                nk = static_cast<T*>(scratch_k);
                nv = static_cast<T*>(scratch_v);
                ck = nk;
                cv = nv;
            }
            launch(s, dim3(heads_total, tiles), dim3(kThreads), smem_in, k_attn_in<T>, x, N, dm, w.attn_norm, w.qkv_w,
                   w.qkv_b, io.positions, m->inv_freq.as<const float>(), q, nk, nv);
            AttnArgs a;
            a.n = n;
            a.ctx = ctx;
            a.B = B;
            a.chunks = chunks;
            a.key_chunk = key_chunk;
            a.cache_seq_stride = size_t(L) * ctx * dm.KV * dm.hd;
            a.mask_mode = mask_mode;
            const bool windowed = m->layer_window[size_t(l)] != 0;
            a.window = mask_mode == kMaskSlots ? (windowed ? window : ctx) : (windowed ? window : 0);
            a.slots = io.slots;
            a.pos0 = io.pos0;
            a.partial = partial;
            a.counters = counters.as<unsigned>();
            const T* bias = static_cast<const T*>(windowed ? io.window_mask : io.mask);
            launch(s, dim3(n, dm.KV, B * chunks), dim3(kThreads), smem_attn, k_attention<T>, q, dm, a, ck, cv,
                   static_cast<const T*>(nk), static_cast<const T*>(nv), bias, w.sinks, attn);
            // The grouped-MoE path's out-projection and router run as one kernel when the widths allow it.
            const bool fused_or = grouped_moe && dm.H * dm.hd == 128 && dm.E <= 2 * kWarps;
            if (!fused_or)
                launch(s, dim3((dm.d + 2 * kWarps - 1) / (2 * kWarps), tiles), dim3(kThreads), smem_out, k_out<T>, attn,
                       x, N, dm, w.out_w, w.out_b, x2);
            if (grouped_moe) {
                int* counts = g_counts.as<int>();
                const unsigned zs = unsigned((N + kGroupRows - 1) / kGroupRows);  // a fully skewed routing still spreads
                if (fused_or)
                    launch(s, dim3(N), dim3(kOrThreads), 0, k_out_route<T>, static_cast<const float*>(attn),
                           static_cast<const float*>(x), N, dm, w, x2, g_xn.as<float>(), ridx, rw,
                           io.routes ? io.routes + size_t(l) * N * dm.k : nullptr, g_lists.as<int>(), counts, err);
                else
                    launch(s, dim3(N), dim3(128), smem_up, k_route_rows<T>, x2, N, dm, w, g_xn.as<float>(), ridx, rw,
                           io.routes ? io.routes + size_t(l) * N * dm.k : nullptr, g_lists.as<int>(), counts, err);
                launch(s, dim3(dm.E, (dm.I + kPairsPerCta - 1) / kPairsPerCta, zs), dim3(kThreads),
                       size_t(kGroupRows) * dm.d * 4, k_moe_up_grouped<T>, static_cast<const float*>(g_xn.as<float>()), N,
                       dm, w, static_cast<const int*>(g_lists.as<int>()), static_cast<const int*>(counts), act);
                launch(s, dim3(dm.E, (dm.d + kWarps - 1) / kWarps, zs), dim3(kThreads), size_t(kGroupRows) * dm.I * 4,
                       k_moe_down_grouped<T>, static_cast<const float*>(act), N, dm, w.w2, w.b2,
                       static_cast<const int*>(g_lists.as<int>()), static_cast<const int*>(counts), g_ys.as<float>());
                launch(s, dim3(N), dim3(std::max(dm.d, dm.E)), 0, k_moe_combine_rows<T>,
                       static_cast<const float*>(g_ys.as<float>()), static_cast<const float*>(x2), N, dm,
                       static_cast<const float*>(rw), x, counts);
                launches += fused_or ? 6 : 7;
                continue;
            }
            launch(s, dim3(N * dm.k, (dm.I + kPairsPerCta - 1) / kPairsPerCta), dim3(kThreads), smem_up, k_moe_up<T>, x2,
                   N, dm, w, ridx, rw, io.routes ? io.routes + size_t(l) * N * dm.k : nullptr, act, err);
            launch(s, dim3(N, (dm.d + kWarps - 1) / kWarps), dim3(kThreads), size_t(dm.k) * dm.I * 4, k_moe_down<T>, act,
                   x2, N, dm, ridx, rw, w.w2, w.b2, x, err);
            launches += 5;
        }
        const int nrows = io.rows ? B : N;
        launch(s, dim3(nrows), dim3(256), 0, k_final_norm<T>, x, nrows, io.rows, n,
               reinterpret_cast<const float*>(m->at(1)), dm, tf, io.keys, err);
        if (!skip_vocab) enqueue_vocab_t<T>(s);
        launches += 2;
        if (side) check(cudaStreamWaitEvent(s, join_ev, 0), "prefetch join");
    }

    // The layers alone, up to the final norm (reads the inputs left by the last run; no L2 prefetch beside them).
    template <typename T> void enqueue_layers_t(cudaStream_t s) {
        if constexpr (std::is_same_v<T, float>) {
            if (cluster_decode) {
                enqueue_cluster_decode(s);
                return;
            }
            if (cluster_fwd) {
                enqueue_cluster_fwd(s);
                return;
            }
        }
        cudaStream_t keep = side;
        side = nullptr;  // enqueue_t without its prefetch fork, then without the vocab kernel
        skip_vocab = true;
        try {
            enqueue_t<T>(s);
        } catch (...) {
            side = keep;
            skip_vocab = false;
            throw;
        }
        side = keep;
        skip_vocab = false;
    }
    void enqueue_layers(cudaStream_t s) {
        if (large_path) throw ValueError("layer-only launches are for the dev-width programs");
        if (m->desc.storage == CHROMA_B200_BF16) enqueue_layers_t<__nv_bfloat16>(s);
        else enqueue_layers_t<float>(s);
    }

    // The vocab projection alone (reads the final-norm rows left by the last run).
    template <typename T> void enqueue_vocab_t(cudaStream_t s) {
        launch_vocab<T>(s, m->dm, sms, tf, io.rows ? B : B * n, reinterpret_cast<const T*>(m->at(2)),
                        static_cast<T*>(io.logits), io.keys, err);
    }

    void enqueue(cudaStream_t s) {
        if (large_path) {
            large.enqueue(s, io, err);
            launches = large.launches;
        } else if (m->desc.storage == CHROMA_B200_BF16) {
            enqueue_t<__nv_bfloat16>(s);
        } else {
            enqueue_t<float>(s);
        }
    }
    void enqueue_vocab(cudaStream_t s) {
        if (large_path) large.enqueue_vocab(s, io, err);
        else if (m->desc.storage == CHROMA_B200_BF16) enqueue_vocab_t<__nv_bfloat16>(s);
        else enqueue_vocab_t<float>(s);
    }
};

// A captured CUDA graph of an enqueue function, rebuilt only when asked.
struct Graph {
    cudaGraphExec_t exec = nullptr;
    bool failed = false;
    ~Graph() {
        if (exec) cudaGraphExecDestroy(exec);
    }
    template <typename F> void run(cudaStream_t s, F&& enqueue) {
        if (!exec && !failed) {
            cudaGraph_t g = nullptr;
            check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
            bool ok = true;
            try {
                enqueue(s);
            } catch (...) {
                ok = false;
            }
            const cudaError_t end = cudaStreamEndCapture(s, &g);
            if (ok && end == cudaSuccess && g && cudaGraphInstantiate(&exec, g, 0) == cudaSuccess) {
                cudaGraphDestroy(g);
            } else {
                if (g) cudaGraphDestroy(g);
                exec = nullptr;
                failed = true;
                cudaGetLastError();
            }
        }
        if (exec) check(cudaGraphLaunch(exec, s), "cudaGraphLaunch");
        else enqueue(s);
    }
};

}  // namespace cb200

using namespace cb200;

struct chroma_b200_program {
    int device = 0;
    std::string name;
    cudaStream_t stream = nullptr;
    std::shared_ptr<Model> model_ptr = std::make_shared<Model>();
    Model& model = *model_ptr;
    GptExec exec;
    std::vector<DevBuf> in, out;
    std::vector<size_t> in_bytes, out_bytes;
    DevBuf err;
    std::unique_ptr<PinnedBuf> err_host;
    DevBuf positions, pos0, routes;
    Graph graph;
    int launches = 0;

    ~chroma_b200_program() {
        if (stream) {
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(device);
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
            cudaSetDevice(prev);
        }
    }

    void enqueue(cudaStream_t s) {
        if (model.desc.kind == CHROMA_B200_MICRO) {
            const auto& d = model.desc;
            const int cols = int(d.cols);
            // Chunks of 8 bf16 per thread; at most 512 threads and 8 chunks per row.
            int chunks = 1;
            while (chunks < 8 && (cols + 8 * chunks - 1) / (8 * chunks) > 256) chunks *= 2;
            int threads = (cols / 8 + chunks - 1) / chunks;
            threads = (threads + 31) / 32 * 32;
            const auto* x = in[0].as<const __nv_bfloat16>();
            const auto* g = in[1].as<const __nv_bfloat16>();
            const auto* u = in[2].as<const __nv_bfloat16>();
            const float* w = reinterpret_cast<const float*>(model.at(0));
            auto* o = out[0].as<__nv_bfloat16>();
            if (chunks == 1) launch(s, dim3(unsigned(d.rows)), dim3(threads), 0, k_micro<1>, x, g, u, w, o, d.rows, cols, d.eps);
            else if (chunks == 2) launch(s, dim3(unsigned(d.rows)), dim3(threads), 0, k_micro<2>, x, g, u, w, o, d.rows, cols, d.eps);
            else if (chunks == 4) launch(s, dim3(unsigned(d.rows)), dim3(threads), 0, k_micro<4>, x, g, u, w, o, d.rows, cols, d.eps);
            else launch(s, dim3(unsigned(d.rows)), dim3(threads), 0, k_micro<8>, x, g, u, w, o, d.rows, cols, d.eps);
            launches = 1;
            return;
        }
        exec.enqueue(s);
        launches = exec.launches;
    }
};

struct chroma_b200_decoder {
    std::shared_ptr<Model> models[2];  // shared with the programs, so either may be destroyed first
    int device = 0, B = 1, ctx = 0, window = 0, L = 0, row = 0, V = 0, steps = 1;
    size_t es = 4;
    cudaStream_t stream = nullptr;
    DevBuf cache_k, cache_v, slots, io_in, commit_pos, positions, last, logits, keys, err;
    int64_t* pos0 = nullptr;    // [B] in io_in, followed by
    int64_t* tokens = nullptr;  // [B][steps]: one host-to-device copy per step uploads both
    std::unique_ptr<PinnedBuf> host_in, host_out, host_commit;
    cudaEvent_t commit_ev = nullptr;  // the last commit's upload of host_commit
    GptExec ex[2];
    DevBuf new_k[2], new_v[2];
    Graph graph[2][2];
    Graph advance_graph;
    DevBuf record, counter;
    int capacity = 0;

    ~chroma_b200_decoder() {
        if (stream) {
            int prev = 0;
            cudaGetDevice(&prev);
            cudaSetDevice(device);
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
            if (commit_ev) cudaEventDestroy(commit_ev);
            cudaSetDevice(prev);
        }
    }
};

namespace {

int fail(char* err, size_t n, int code, const char* msg) {
    if (err && n) {
        std::snprintf(err, n, "%s", msg);
    }
    return code;
}

template <typename F> int guarded(char* err, size_t n, F&& f) {
    try {
        f();
        return CHROMA_B200_OK;
    } catch (const IndexError& e) {
        return fail(err, n, CHROMA_B200_INDEX, e.what());
    } catch (const ValueError& e) {
        return fail(err, n, CHROMA_B200_VALUE, e.what());
    } catch (const std::exception& e) {
        return fail(err, n, CHROMA_B200_RUNTIME, e.what());
    } catch (...) {
        return fail(err, n, CHROMA_B200_RUNTIME, "unknown native error");
    }
}

// The device error word after a call: an out-of-range index (IndexError, as runtime.h:160-162), or a bounded
// wait that gave up (a TMA/tensor-core pipeline stage, or another rank of an expert-parallel group that did not
// arrive).
void raise_device_errors(unsigned word) {
    if (word & kErrIndex) throw IndexError("Tensor index out of range");
    if (word & kErrTimeout)
        throw std::runtime_error("a bounded device wait timed out (an expert-parallel rank did not arrive, or a "
                                 "pipeline stage stalled); expert-parallel groups must be recreated after this");
}

void read_error_word(cudaStream_t s, DevBuf& err, unsigned* host) {
    check(cudaMemcpyAsync(host, err.p, sizeof(unsigned), cudaMemcpyDeviceToHost, s), "Read index error");
    check(cudaStreamSynchronize(s), "CUDA execution");
    raise_device_errors(*host);
}

}  // namespace

extern "C" {

static void create_program(const chroma_b200_desc* desc, const char* weights_path, const void* device_weights,
                           chroma_b200_program** out, std::shared_ptr<EpGroup> ep = nullptr);

int chroma_b200_create(const chroma_b200_desc* desc, const char* weights_path, chroma_b200_program** out, char* err,
                       size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!desc || !weights_path || !out) throw ValueError("null argument");
        create_program(desc, weights_path, nullptr, out);
    });
}

int chroma_b200_create_device(const chroma_b200_desc* desc, const void* device_weights, chroma_b200_program** out,
                              char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!desc || !device_weights || !out) throw ValueError("null argument");
        create_program(desc, nullptr, device_weights, out);
    });
}

struct chroma_b200_ep {
    std::shared_ptr<EpGroup> group;
};

int chroma_b200_ep_create(int32_t rank, int32_t world, int64_t max_pairs, int32_t hidden, int32_t experts,
                          int32_t vocab_rows, int32_t vocab, chroma_b200_ep** out, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!out) throw ValueError("null argument");
        if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world)
            throw ValueError("expert-parallel rank/world out of range (world <= 8)");
        if (experts < 1 || experts > kEpMaxExperts || experts % world)
            throw ValueError("experts must divide evenly over the group (at most 256)");
        if (hidden < 8 || hidden % 8 || max_pairs < 1 || max_pairs > (int64_t(1) << 31) / world)
            throw ValueError("expert-parallel buffer shape out of range");
        auto g = std::make_shared<EpGroup>();
        check(cudaGetDevice(&g->device), "cudaGetDevice");
        g->rank = rank;
        g->world = world;
        g->E = experts;
        g->d = hidden;
        g->pmax = max_pairs;
        g->cap = max_pairs * world;
        auto align = [](size_t b) { return (b + 1023) / 1024 * 1024; };
        g->off_meta = align(sizeof(EpHeader));
        g->off_x = g->off_meta + align(size_t(g->cap) * 4);
        g->off_y = g->off_x + align(size_t(g->cap) * hidden * 2);
        size_t bytes = g->off_y + align(size_t(max_pairs) * hidden * 2);
        if (vocab_rows > 0) {
            if (vocab < world || vocab % 8) throw ValueError("vocab shard needs a vocab that is a multiple of 8");
            g->vrows_max = vocab_rows;
            g->V = vocab;
            g->Vl = (vocab + world - 1) / world;
            g->off_vrows = bytes;
            g->off_vkeys = g->off_vrows + align(size_t(world) * vocab_rows * hidden * 2);
            g->off_vlogits = g->off_vkeys + align(size_t(world) * vocab_rows * 8);
            bytes = g->off_vlogits + align(size_t(vocab_rows) * vocab * 2);
        }
        g->shared = DevBuf(bytes);
        check(cudaMemset(g->shared.p, 0, g->off_x), "expert-parallel header");
        g->local = DevBuf(256);
        check(cudaMemset(g->local.p, 0, 256), "expert-parallel counters");
        check(cudaDeviceSynchronize(), "expert-parallel init");
        g->peer[size_t(rank)] = g->shared.as<char>();
        if (const char* ms = std::getenv("CHROMA_B200_EP_TIMEOUT_MS")) {
            const long long v = std::atoll(ms);
            if (v > 0) g->timeout_ns = (unsigned long long)v * 1000000ull;
        }
        *out = new chroma_b200_ep{std::move(g)};
    });
}

int chroma_b200_ep_handle(const chroma_b200_ep* ep, void* handle, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!ep || !handle) throw ValueError("null argument");
        cudaIpcMemHandle_t h;
        check(cudaIpcGetMemHandle(&h, ep->group->shared.p), "cudaIpcGetMemHandle");
        std::memcpy(handle, &h, sizeof(h));
    });
}

int chroma_b200_ep_open(chroma_b200_ep* ep, const void* handles, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!ep || !handles) throw ValueError("null argument");
        EpGroup& g = *ep->group;
        if (g.open) throw ValueError("expert-parallel group already open");
        const char* h = static_cast<const char*>(handles);
        for (int q = 0; q < g.world; ++q) {
            if (q == g.rank) continue;
            cudaIpcMemHandle_t mh;
            std::memcpy(&mh, h + size_t(q) * sizeof(mh), sizeof(mh));
            void* ptr = nullptr;
            check(cudaIpcOpenMemHandle(&ptr, mh, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
            g.opened.push_back(ptr);
            g.peer[size_t(q)] = static_cast<char*>(ptr);
        }
        g.open = true;
    });
}

void chroma_b200_ep_destroy(chroma_b200_ep* ep) { delete ep; }

int chroma_b200_create_ep(const chroma_b200_desc* desc, const char* weights_path, const void* device_weights,
                          chroma_b200_ep* ep, chroma_b200_program** out, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!desc || !ep || !out || (weights_path == nullptr) == (device_weights == nullptr))
            throw ValueError("null argument (exactly one of weights_path / device_weights)");
        create_program(desc, weights_path, device_weights, out, ep->group);
    });
}

}  // extern "C"

static void create_program(const chroma_b200_desc* desc, const char* weights_path, const void* device_weights,
                           chroma_b200_program** out, std::shared_ptr<EpGroup> ep) {
    {
        validate_desc(*desc);
        if (ep) {
            if (!ep->open) throw ValueError("expert-parallel group not opened (exchange the handles first)");
            if (!is_large(*desc) || desc->kind == CHROMA_B200_MICRO)
                throw ValueError("expert parallelism needs a large-width bf16 GPT-OSS program (hidden >= 1024, head_dim 64)");
            if (desc->experts != ep->E || desc->hidden != ep->d)
                throw ValueError("program and expert-parallel group disagree on experts / hidden size");
            int dev = 0;
            check(cudaGetDevice(&dev), "cudaGetDevice");
            if (dev != ep->device) throw ValueError("expert-parallel group lives on another device");
        }
        auto p = std::make_unique<chroma_b200_program>();
        check(cudaGetDevice(&p->device), "cudaGetDevice");
        cudaDeviceProp prop{};
        check(cudaGetDeviceProperties(&prop, p->device), "cudaGetDeviceProperties");
        if (prop.major != 10)
            throw std::runtime_error(std::string("chroma_b200 kernels are built for sm_100a (B200); found ") + prop.name);
        p->name = prop.name;
        Model& m = p->model;
        m.desc = *desc;
        m.device = p->device;
        m.ep = ep;
        m.El = ep ? desc->experts / ep->world : desc->experts;
        m.offsets.assign(desc->offsets, desc->offsets + desc->num_offsets);
        for (int64_t off : m.offsets)
            if (off < 0 || off >= desc->weight_bytes || off % 16) throw ValueError("weight offset out of range or unaligned");
        if (weights_path) {
            m.weights = load_weights(weights_path, size_t(desc->weight_bytes), p->device);
        } else {
            m.weights = std::make_shared<Weights>();
            m.weights->device = p->device;
            m.weights->ptr = static_cast<const char*>(device_weights);
        }
        m.desc.offsets = nullptr;
        m.desc.inv_freq = nullptr;
        m.desc.layer_window = nullptr;
        check(cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        p->err = DevBuf(sizeof(unsigned));
        p->err_host = std::make_unique<PinnedBuf>(sizeof(unsigned));
        check(cudaMemset(p->err.p, 0, sizeof(unsigned)), "cudaMemset");
        const auto& d = *desc;
        if (d.kind == CHROMA_B200_MICRO) {
            const size_t bytes = size_t(d.rows) * size_t(d.cols) * 2;
            for (int i = 0; i < 3; ++i) {
                p->in.emplace_back(bytes);
                p->in_bytes.push_back(bytes);
            }
            p->out.emplace_back(bytes);
            p->out_bytes.push_back(bytes);
        } else {
            Dims& dm = m.dm;
            dm.d = d.hidden;
            dm.H = d.heads;
            dm.KV = d.kv_heads;
            dm.hd = d.head_dim;
            dm.G = d.heads / d.kv_heads;
            dm.E = d.experts;
            dm.k = d.top_k;
            dm.I = d.intermediate;
            dm.V = d.vocab;
            dm.eps = d.eps;
            dm.sm_scale = d.sm_scale;
            dm.alpha = d.swiglu_alpha;
            dm.limit = d.swiglu_limit;
            dm.conc = d.rope_concentration;
            m.layer_window.assign(desc->layer_window, desc->layer_window + d.layers);
            m.inv_freq = DevBuf(size_t(d.head_dim / 2) * 4);
            check(cudaMemcpy(m.inv_freq.p, desc->inv_freq, size_t(d.head_dim / 2) * 4, cudaMemcpyHostToDevice), "rope table");
            const size_t es = storage_size(d.storage);
            const size_t n = size_t(d.tokens);
            const size_t V = size_t(d.vocab);
            const size_t cache = size_t(d.layers) * d.context * d.kv_heads * d.head_dim * es;
            const size_t rows_kv = size_t(d.layers) * n * d.kv_heads * d.head_dim * es;
            GptIO& io = p->exec.io;
            if (d.kind == CHROMA_B200_GPTOSS_CACHED) {
                const size_t mask = n * (d.context + n) * es;
                const size_t sizes[7] = {n * 8, n * 4, cache, cache, mask, mask, 8};
                for (size_t b : sizes) {
                    p->in.emplace_back(b);
                    p->in_bytes.push_back(b);
                }
                const size_t osz[3] = {V * es, rows_kv, rows_kv};
                for (size_t b : osz) {
                    p->out.emplace_back(b);
                    p->out_bytes.push_back(b);
                }
                p->exec.init(m, 1, int(n), d.context, kMaskBuffer, d.window, true);
                io.tokens = p->in[0].as<const int64_t>();
                io.positions = p->in[1].as<const float>();
                io.cache_k = p->in[2].p;
                io.cache_v = p->in[3].p;
                io.mask = p->in[4].p;
                io.window_mask = p->in[5].p;
                io.rows = p->in[6].as<const int64_t>();
                io.logits = p->out[0].p;
                io.new_k = p->out[1].p;
                io.new_v = p->out[2].p;
            } else {
                p->in.emplace_back(n * 8);
                p->in_bytes.push_back(n * 8);
                const bool last = d.kind == CHROMA_B200_GPTOSS_LAST;
                if (last) {
                    p->in.emplace_back(8);
                    p->in_bytes.push_back(8);
                }
                const size_t ob = (last ? 1 : n) * V * es;
                p->out.emplace_back(ob);
                p->out_bytes.push_back(ob);
                p->exec.init(m, 1, int(n), 0, kMaskCausal, d.window, last);
                p->positions = DevBuf(n * 4);
                std::vector<float> pos(n);
                for (size_t i = 0; i < n; ++i) pos[i] = float(i);
                check(cudaMemcpy(p->positions.p, pos.data(), n * 4, cudaMemcpyHostToDevice), "positions");
                io.tokens = p->in[0].as<const int64_t>();
                io.positions = p->positions.as<const float>();
                io.rows = last ? p->in[1].as<const int64_t>() : nullptr;
                io.logits = p->out[0].p;
            }
            p->exec.err = p->err.as<unsigned>();
            p->routes = DevBuf(size_t(d.layers) * n * d.top_k * 4);
            check(cudaMemset(p->routes.p, 0xff, p->routes.bytes), "routes");
            io.routes = p->routes.as<int>();
        }
        check(cudaDeviceSynchronize(), "create");
        *out = p.release();
    }
}

extern "C" {

int chroma_b200_run(chroma_b200_program* p, const void* const* inputs, void* const* outputs, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!p) throw ValueError("null program");
        DeviceGuard guard(p->device);
        unsigned* eh = static_cast<unsigned*>(p->err_host->p);
        try {
            check(cudaMemsetAsync(p->err.p, 0, sizeof(unsigned), p->stream), "Reset index error");
            for (size_t i = 0; i < p->in.size(); ++i)
                check(cudaMemcpyAsync(p->in[i].p, inputs[i], p->in_bytes[i], cudaMemcpyHostToDevice, p->stream),
                      "Upload input");
            p->graph.run(p->stream, [&](cudaStream_t s) { p->enqueue(s); });
            read_error_word(p->stream, p->err, eh);
            for (size_t i = 0; i < p->out.size(); ++i)
                check(cudaMemcpyAsync(outputs[i], p->out[i].p, p->out_bytes[i], cudaMemcpyDeviceToHost, p->stream),
                      "Download output");
            check(cudaStreamSynchronize(p->stream), "Download output");
        } catch (...) {
            // Host buffers must outlive every queued transfer (runtime.h:168-172).
            cudaStreamSynchronize(p->stream);
            throw;
        }
    });
}

int chroma_b200_buffers(chroma_b200_program* p, void** inputs, void** outputs, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!p) throw ValueError("null program");
        for (size_t i = 0; i < p->in.size(); ++i)
            if (inputs) inputs[i] = p->in[i].p;
        for (size_t i = 0; i < p->out.size(); ++i)
            if (outputs) outputs[i] = p->out[i].p;
    });
}

int chroma_b200_run_device(chroma_b200_program* p, void* stream, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!p) throw ValueError("null program");
        DeviceGuard guard(p->device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : p->stream;
        p->graph.run(s, [&](cudaStream_t st) { p->enqueue(st); });
    });
}

int chroma_b200_check(chroma_b200_program* p, void* stream, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!p) throw ValueError("null program");
        DeviceGuard guard(p->device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : p->stream;
        unsigned* eh = static_cast<unsigned*>(p->err_host->p);
        check(cudaMemcpyAsync(eh, p->err.p, sizeof(unsigned), cudaMemcpyDeviceToHost, s), "Read index error");
        check(cudaMemsetAsync(p->err.p, 0, sizeof(unsigned), s), "Reset index error");
        check(cudaStreamSynchronize(s), "CUDA execution");
        raise_device_errors(*eh);
    });
}

const char* chroma_b200_device(const chroma_b200_program* p) { return p ? p->name.c_str() : ""; }

int32_t chroma_b200_launches(const chroma_b200_program* p) { return p ? p->launches : 0; }

void chroma_b200_destroy(chroma_b200_program* p) { delete p; }

int64_t chroma_b200_plan_arena(int32_t count, const int64_t* sizes, const int32_t* starts, const int32_t* ends,
                               int64_t* offsets) {
    if (count < 0 || (count > 0 && (!sizes || !starts || !ends || !offsets))) return -1;
    std::vector<Alloc> a(static_cast<size_t>(count));
    for (int32_t i = 0; i < count; ++i) a[size_t(i)] = {size_t(sizes[i]), starts[i], ends[i], 0};
    const size_t total = plan_arena(a);
    for (int32_t i = 0; i < count; ++i) offsets[i] = int64_t(a[size_t(i)].offset);
    return int64_t(total);
}

int chroma_b200_routes(chroma_b200_program* p, int32_t* out, int64_t count, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!p || !out) throw ValueError("null argument");
        if (!p->routes.p || size_t(count) * 4 != p->routes.bytes) throw ValueError("routes buffer size mismatch");
        DeviceGuard guard(p->device);
        check(cudaMemcpyAsync(out, p->routes.p, p->routes.bytes, cudaMemcpyDeviceToHost, p->stream), "routes");
        check(cudaStreamSynchronize(p->stream), "routes");
    });
}

// ---------------------------------------------------------------------------------------------------------
// Vocab projection + greedy argmax that allocates nothing. For callers that cannot call cudaMalloc: code running
// inside a stream capture another framework owns, allocator-free embedded runtimes, or hosts that hand this library
// pre-sized device buffers and forbid it from touching the allocator. The only scratch (one 64-bit argmax key per
// row) lives in the static array below, kStaticArgmaxRows entries, which every GPU that loads this library holds
// until exit.
constexpr int kStaticArgmaxRows = 256;
static __device__ __align__(256) unsigned long long g_static_argmax_keys[kStaticArgmaxRows];

__global__ void k_clear_keys(unsigned long long* keys, int rows) {
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < rows; i += blockDim.x) keys[i] = 0ull;
}

__global__ void k_keys_to_ids(const unsigned long long* keys, int rows, int64_t* ids) {
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < rows; i += blockDim.x) ids[i] = argmax_index(keys[i]);
}

// Device address of the static scratch, looked up once per device (with that device current). In host code the
// array's name is only a host-side stand-in, never a device address.
constexpr int kMaxDevices = 64;
static std::mutex g_static_mu;
static unsigned long long* g_static_keys[kMaxDevices] = {};

static unsigned long long* static_keys(int device) {
    if (device < 0 || device >= kMaxDevices) throw std::runtime_error("device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_keys[device]) {
        unsigned long long* ptr = nullptr;
        check(cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_static_argmax_keys), "cudaGetSymbolAddress");
        g_static_keys[device] = ptr;
    }
    return g_static_keys[device];
}

int chroma_b200_vocab_argmax_static(const chroma_b200_program* p, const float* x, int32_t rows, void* logits,
                                    int64_t* ids, void* stream, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!p || !x || !ids) throw ValueError("null argument");
        const auto& d = p->model.desc;
        if (d.kind == CHROMA_B200_MICRO) throw ValueError("not a GPT-OSS program");
        // A vocab-sharded expert-parallel program holds only its rank's unembedding rows.
        if (p->model.ep && p->model.ep->vrows_max > 0)
            throw ValueError("vocab-sharded program: it holds only its rank's unembedding rows");
        if (rows < 1 || rows > kStaticArgmaxRows)
            throw ValueError("rows must be in [1, " + std::to_string(kStaticArgmaxRows) +
                             "]: the static argmax scratch holds that many rows");
        DeviceGuard guard(p->device);
        unsigned long long* keys = static_keys(p->device);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const Dims& dm = p->model.dm;
        launch(s, dim3(1), dim3(256), 0, k_clear_keys, keys, int(rows));
        if (d.storage == CHROMA_B200_BF16)
            launch_vocab<__nv_bfloat16>(s, dm, p->exec.sms, x, int(rows),
                                        reinterpret_cast<const __nv_bfloat16*>(p->model.at(2)),
                                        static_cast<__nv_bfloat16*>(logits), keys, p->err.as<unsigned>(), false);
        else
            launch_vocab<float>(s, dm, p->exec.sms, x, int(rows), reinterpret_cast<const float*>(p->model.at(2)),
                                static_cast<float*>(logits), keys, p->err.as<unsigned>(), false);
        launch(s, dim3(1), dim3(256), 0, k_keys_to_ids, keys, int(rows), ids);
    });
}

int chroma_b200_gemm_bf16(const void* a, const void* b, const void* bias, const void* residual, void* c, int32_t m,
                          int32_t n, int32_t k, int32_t epilogue, float swiglu_alpha, float swiglu_limit, int32_t groups,
                          const int32_t* offsets, void* tile_scratch, unsigned int* error_word, void* stream, char* err,
                          size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!a || !b || !c || !error_word) throw ValueError("null argument");
        if (m < 1 || n < 1 || k < 1) throw ValueError("GEMM sizes must be positive");
        if (epilogue < kEpiStore || epilogue > kEpiExpert) throw ValueError("unknown GEMM epilogue");
        if (epilogue == kEpiResidual && !residual) throw ValueError("residual epilogue needs the residual matrix");
        int dev = 0, sms = 148;
        check(cudaGetDevice(&dev), "cudaGetDevice");
        check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
        GemmArgs g{};
        g.M = m;
        g.N = n;
        g.K = k;
        g.epi = epilogue;
        g.bias = static_cast<const __nv_bfloat16*>(bias);
        g.residual = static_cast<const __nv_bfloat16*>(residual);
        g.ldr = n;
        g.C = static_cast<__nv_bfloat16*>(c);
        g.ldc = epilogue == kEpiSwiglu ? n / 2 : n;
        g.alpha = swiglu_alpha;
        g.limit = swiglu_limit;
        g.groups = groups;
        g.offsets = offsets;
        gemm_bf16(static_cast<cudaStream_t>(stream), a, b, g, m, groups * n, tile_scratch, sms, error_word);
    });
}

int64_t chroma_b200_workspace_bytes(const chroma_b200_program* p) { return p ? int64_t(p->exec.arena_bytes) : 0; }

// ---------------------------------------------------------------------------------------------------------
int chroma_b200_decoder_create(chroma_b200_program* prefill, chroma_b200_program* decode, int32_t sliding_window,
                               int32_t batch, chroma_b200_decoder** out, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!prefill || !decode || !out) throw ValueError("null argument");
        const auto& pd = prefill->model.desc;
        const auto& dd = decode->model.desc;
        if (pd.kind != CHROMA_B200_GPTOSS_CACHED || dd.kind != CHROMA_B200_GPTOSS_CACHED || dd.tokens != 1 ||
            pd.context != dd.context || pd.layers != dd.layers || pd.vocab != dd.vocab || pd.storage != dd.storage ||
            pd.tokens < 1 || pd.tokens > pd.context)
            throw ValueError("Decoder prefill and decode were not exported as a pair");
        if (batch < 1) throw ValueError("batch must be positive");
        if (sliding_window < 0) throw ValueError("sliding_window must be nonnegative");
        DeviceGuard guard(decode->device);
        auto d = std::make_unique<chroma_b200_decoder>();
        d->models[0] = prefill->model_ptr;
        d->models[1] = decode->model_ptr;
        d->device = decode->device;
        d->B = batch;
        d->ctx = dd.context;
        d->window = sliding_window > 0 ? std::min(sliding_window, dd.context) : dd.context;
        d->L = dd.layers;
        d->row = dd.kv_heads * dd.head_dim;
        d->V = dd.vocab;
        d->steps = pd.tokens;
        d->es = storage_size(dd.storage);
        check(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        const size_t cache = size_t(batch) * d->L * d->ctx * d->row * d->es;
        d->cache_k = DevBuf(cache);
        d->cache_v = DevBuf(cache);
        check(cudaMemset(d->cache_k.p, 0, cache), "cache");
        check(cudaMemset(d->cache_v.p, 0, cache), "cache");
        d->slots = DevBuf(size_t(batch) * d->ctx * 8);
        check(cudaMemset(d->slots.p, 0xff, size_t(batch) * d->ctx * 8), "slots");
        d->io_in = DevBuf(size_t(batch) * (d->steps + 1) * 8);
        d->pos0 = d->io_in.as<int64_t>();
        d->tokens = d->pos0 + batch;
        d->commit_pos = DevBuf(size_t(batch) * 8);
        d->positions = DevBuf(size_t(batch) * d->steps * 4);
        d->last = DevBuf(size_t(batch) * 8);
        d->logits = DevBuf(size_t(batch) * d->V * d->es);
        d->keys = DevBuf(size_t(batch) * 8);
        d->err = DevBuf(sizeof(unsigned));
        check(cudaMemset(d->err.p, 0, sizeof(unsigned)), "cudaMemset");
        d->host_in = std::make_unique<PinnedBuf>(size_t(batch) * (d->steps + 1) * 8);
        d->host_out = std::make_unique<PinnedBuf>(size_t(batch) * 8 + 16);
        d->host_commit = std::make_unique<PinnedBuf>(size_t(batch) * 8);
        check(cudaEventCreateWithFlags(&d->commit_ev, cudaEventDisableTiming), "commit event");
        for (int i = 0; i < 2; ++i) {
            const int n = d->models[i]->desc.tokens;
            const size_t staged = size_t(d->L) * batch * n * d->row * d->es;
            d->new_k[i] = DevBuf(staged);
            d->new_v[i] = DevBuf(staged);
            GptExec& e = d->ex[i];
            e.init(*d->models[i], batch, n, d->ctx, kMaskSlots, d->window, true);
            e.err = d->err.as<unsigned>();
            e.io.tokens = d->tokens;
            e.io.positions = d->positions.as<const float>();
            e.io.cache_k = d->cache_k.p;
            e.io.cache_v = d->cache_v.p;
            e.io.new_k = d->new_k[i].p;
            e.io.new_v = d->new_v[i].p;
            e.io.slots = d->slots.as<const int64_t>();
            e.io.pos0 = d->pos0;
            e.io.rows = d->last.as<const int64_t>();
            e.io.logits = d->logits.p;
            e.io.keys = nullptr;
        }
        check(cudaDeviceSynchronize(), "decoder create");
        *out = d.release();
    });
}

int chroma_b200_decoder_step(chroma_b200_decoder* d, int32_t use_decode, const int64_t* tokens, int32_t count,
                             const int64_t* positions, void* logits, int64_t* argmax, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d || !tokens || !positions) throw ValueError("null argument");
        const int which = use_decode ? 1 : 0;
        GptExec& e = d->ex[which];
        const int n = e.n;
        if (count < 1 || count > n) throw ValueError("count out of range for this program");
        DeviceGuard guard(d->device);
        cudaStream_t s = d->stream;
        int64_t* hin = static_cast<int64_t*>(d->host_in->p);
        std::memcpy(hin, positions, size_t(d->B) * 8);
        std::memcpy(hin + d->B, tokens, size_t(d->B) * n * 8);
        try {
            check(cudaMemcpyAsync(d->pos0, hin, size_t(d->B) * (n + 1) * 8, cudaMemcpyHostToDevice, s),
                  "Upload positions and tokens");
            launch(s, dim3((d->B * n + 255) / 256), dim3(256), 0, k_positions, static_cast<const int64_t*>(d->pos0), d->B,
                   n, d->positions.as<float>(), d->last.as<int64_t>(), count, d->err.as<unsigned>());
            // The argmax flag changes the kernel arguments, so each (program, argmax) pair has its own captured graph.
            e.io.keys = argmax ? d->keys.as<unsigned long long>() : nullptr;
            d->graph[which][argmax ? 1 : 0].run(s, [&](cudaStream_t st) { e.enqueue(st); });
            unsigned* eh = static_cast<unsigned*>(d->host_out->p);
            int64_t* am = reinterpret_cast<int64_t*>(static_cast<char*>(d->host_out->p) + 16);
            check(cudaMemcpyAsync(eh, d->err.p, sizeof(unsigned), cudaMemcpyDeviceToHost, s), "Read index error");
            if (argmax)
                check(cudaMemcpyAsync(am, d->keys.p, size_t(d->B) * 8, cudaMemcpyDeviceToHost, s), "Download argmax");
            if (logits)
                check(cudaMemcpyAsync(logits, d->logits.p, size_t(d->B) * d->V * d->es, cudaMemcpyDeviceToHost, s),
                      "Download logits");
            check(cudaStreamSynchronize(s), "CUDA execution");
            raise_device_errors(*eh);
            if (argmax)
                for (int b = 0; b < d->B; ++b) argmax[b] = argmax_index(static_cast<unsigned long long>(am[b]));
        } catch (...) {
            cudaStreamSynchronize(s);
            throw;
        }
    });
}

int chroma_b200_decoder_commit(chroma_b200_decoder* d, int32_t use_decode, int32_t count, const int64_t* positions,
                               char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d || !positions) throw ValueError("null argument");
        const int which = use_decode ? 1 : 0;
        const GptExec& e = d->ex[which];
        if (count < 1 || count > e.n) throw ValueError("count out of range for this program");
        DeviceGuard guard(d->device);
        // Re-upload the chunk's positions: committing is idempotent and independent of later steps' pos0. The commit
        // is only enqueued (everything that reads the caches runs on the same stream); its pinned upload buffer is
        // reused once the previous commit's copy has completed.
        check(cudaEventSynchronize(d->commit_ev), "commit buffer");
        int64_t* hin = static_cast<int64_t*>(d->host_commit->p);
        std::memcpy(hin, positions, size_t(d->B) * 8);
        check(cudaMemcpyAsync(d->commit_pos.p, hin, size_t(d->B) * 8, cudaMemcpyHostToDevice, d->stream), "commit positions");
        check(cudaEventRecord(d->commit_ev, d->stream), "commit event");
        const dim3 grid(unsigned(d->L * d->B * count));
        const int threads = std::min(256, ((d->row + 31) / 32) * 32);
        if (d->es == 2)
            launch(d->stream, grid, dim3(threads), 0, k_commit<__nv_bfloat16>, d->new_k[which].as<const __nv_bfloat16>(),
                   d->new_v[which].as<const __nv_bfloat16>(), d->L, d->B, e.n, count, d->ctx, d->row, 1,
                   d->commit_pos.as<const int64_t>(), d->cache_k.as<__nv_bfloat16>(), d->cache_v.as<__nv_bfloat16>(),
                   d->slots.as<int64_t>());
        else
            launch(d->stream, grid, dim3(threads), 0, k_commit<float>, d->new_k[which].as<const float>(),
                   d->new_v[which].as<const float>(), d->L, d->B, e.n, count, d->ctx, d->row, 1,
                   d->commit_pos.as<const int64_t>(), d->cache_k.as<float>(), d->cache_v.as<float>(), d->slots.as<int64_t>());
    });
}

int chroma_b200_decoder_advance(chroma_b200_decoder* d, const int64_t* tokens, const int64_t* positions, int32_t steps,
                                void* stream, int64_t* ids, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d) throw ValueError("null decoder");
        if (steps < 1) throw ValueError("steps must be positive");
        if ((tokens == nullptr) != (positions == nullptr)) throw ValueError("tokens and positions go together");
        DeviceGuard guard(d->device);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : d->stream;
        if (tokens) {
            int64_t* hin = static_cast<int64_t*>(d->host_in->p);
            check(cudaStreamSynchronize(s), "advance");
            std::memcpy(hin, positions, size_t(d->B) * 8);
            std::memcpy(hin + d->B, tokens, size_t(d->B) * 8);
            check(cudaMemcpyAsync(d->pos0, hin, size_t(d->B) * 16, cudaMemcpyHostToDevice, s), "advance positions and tokens");
        }
        if (!d->record.p || d->capacity < steps) {
            check(cudaStreamSynchronize(s), "advance");
            d->capacity = std::max(steps, 1024);
            d->record = DevBuf(size_t(d->capacity) * d->B * 8);
            d->counter = DevBuf(sizeof(int));
            d->advance_graph = Graph();
        }
        check(cudaMemsetAsync(d->counter.p, 0, sizeof(int), s), "advance counter");
        check(cudaMemsetAsync(d->err.p, 0, sizeof(unsigned), s), "Reset index error");
        GptExec& e = d->ex[1];
        for (int i = 0; i < steps; ++i) {
            d->advance_graph.run(s, [&](cudaStream_t st) {
                e.io.keys = d->keys.as<unsigned long long>();
                if (e.cluster_decode) {
                    // One cluster launch computes the positions itself and commits its rows in place.
                    e.io.commit_k = d->cache_k.p;
                    e.io.commit_v = d->cache_v.p;
                    e.io.commit_slots = d->slots.as<int64_t>();
                    e.enqueue(st);
                    e.io.commit_k = e.io.commit_v = nullptr;
                    e.io.commit_slots = nullptr;
                    launch(st, dim3(1), dim3(std::min(1024, ((d->B + 31) / 32) * 32)), 0, k_advance,
                           d->keys.as<const unsigned long long>(), d->B, d->tokens, d->pos0, d->record.as<int64_t>(),
                           d->counter.as<int>(), d->capacity);
                    return;
                }
                launch(st, dim3((d->B + 255) / 256), dim3(256), 0, k_positions, static_cast<const int64_t*>(d->pos0), d->B,
                       1, d->positions.as<float>(), d->last.as<int64_t>(), 1, static_cast<unsigned*>(nullptr));
                e.enqueue(st);
                const dim3 grid(unsigned(d->L * d->B));
                const int threads = std::min(256, ((d->row + 31) / 32) * 32);
                if (d->es == 2)
                    launch(st, grid, dim3(threads), 0, k_commit<__nv_bfloat16>, d->new_k[1].as<const __nv_bfloat16>(),
                           d->new_v[1].as<const __nv_bfloat16>(), d->L, d->B, 1, 1, d->ctx, d->row, 1,
                           static_cast<const int64_t*>(d->pos0), d->cache_k.as<__nv_bfloat16>(), d->cache_v.as<__nv_bfloat16>(),
                           d->slots.as<int64_t>());
                else
                    launch(st, grid, dim3(threads), 0, k_commit<float>, d->new_k[1].as<const float>(),
                           d->new_v[1].as<const float>(), d->L, d->B, 1, 1, d->ctx, d->row, 1,
                           static_cast<const int64_t*>(d->pos0), d->cache_k.as<float>(), d->cache_v.as<float>(),
                           d->slots.as<int64_t>());
                launch(st, dim3(1), dim3(std::min(1024, ((d->B + 31) / 32) * 32)), 0, k_advance,
                       d->keys.as<const unsigned long long>(), d->B, d->tokens, d->pos0,
                       d->record.as<int64_t>(), d->counter.as<int>(), d->capacity);
            });
        }
        if (ids) {
            unsigned* eh = static_cast<unsigned*>(d->host_out->p);
            check(cudaMemcpyAsync(ids, d->record.p, size_t(steps) * d->B * 8, cudaMemcpyDeviceToHost, s), "advance ids");
            check(cudaMemcpyAsync(eh, d->err.p, sizeof(unsigned), cudaMemcpyDeviceToHost, s), "Read index error");
            check(cudaStreamSynchronize(s), "advance");
            raise_device_errors(*eh);
        }
    });
}

int32_t chroma_b200_decoder_step_launches(const chroma_b200_decoder* d) {
    // positions + decode program (with its L2 prefetch) + commit + advance; the cluster path commits in place and
    // derives the position itself
    if (!d) return 0;
    return d->ex[1].cluster_decode ? d->ex[1].planned_launches() + 1 : 1 + d->ex[1].planned_launches() + 2;
}

int chroma_b200_decoder_launch_layers(chroma_b200_decoder* d, void* stream, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d) throw ValueError("null decoder");
        DeviceGuard guard(d->device);
        d->ex[1].enqueue_layers(stream ? static_cast<cudaStream_t>(stream) : d->stream);
    });
}

int chroma_b200_decoder_launch_vocab(chroma_b200_decoder* d, void* stream, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d) throw ValueError("null decoder");
        DeviceGuard guard(d->device);
        d->ex[1].enqueue_vocab(stream ? static_cast<cudaStream_t>(stream) : d->stream);
    });
}

int chroma_b200_decoder_reset(chroma_b200_decoder* d, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d) throw ValueError("null decoder");
        DeviceGuard guard(d->device);
        check(cudaMemsetAsync(d->slots.p, 0xff, size_t(d->B) * d->ctx * 8, d->stream), "reset");
        check(cudaMemsetAsync(d->cache_k.p, 0, d->cache_k.bytes, d->stream), "reset");
        check(cudaMemsetAsync(d->cache_v.p, 0, d->cache_v.bytes, d->stream), "reset");
        check(cudaStreamSynchronize(d->stream), "reset");
    });
}

int chroma_b200_decoder_read(chroma_b200_decoder* d, void* keys, void* values, int64_t* slots, char* err,
                             size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d) throw ValueError("null decoder");
        DeviceGuard guard(d->device);
        if (keys) check(cudaMemcpyAsync(keys, d->cache_k.p, d->cache_k.bytes, cudaMemcpyDeviceToHost, d->stream), "read");
        if (values) check(cudaMemcpyAsync(values, d->cache_v.p, d->cache_v.bytes, cudaMemcpyDeviceToHost, d->stream), "read");
        if (slots) check(cudaMemcpyAsync(slots, d->slots.p, d->slots.bytes, cudaMemcpyDeviceToHost, d->stream), "read");
        check(cudaStreamSynchronize(d->stream), "read");
    });
}

int chroma_b200_decoder_write(chroma_b200_decoder* d, int32_t first, int32_t count, const void* keys,
                              const void* values, const int64_t* slots, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!d || !keys || !values || !slots) throw ValueError("null argument");
        if (first < 0 || count < 1 || first + count > d->B) throw ValueError("sequence range outside the batch");
        DeviceGuard guard(d->device);
        const size_t per_seq = d->cache_k.bytes / size_t(d->B);
        const size_t slot_bytes = size_t(d->ctx) * 8;
        char* ck = d->cache_k.as<char>() + size_t(first) * per_seq;
        char* cv = d->cache_v.as<char>() + size_t(first) * per_seq;
        check(cudaMemcpyAsync(ck, keys, size_t(count) * per_seq, cudaMemcpyDefault, d->stream), "write keys");
        check(cudaMemcpyAsync(cv, values, size_t(count) * per_seq, cudaMemcpyDefault, d->stream), "write values");
        check(cudaMemcpyAsync(d->slots.as<char>() + size_t(first) * slot_bytes, slots, size_t(count) * slot_bytes,
                              cudaMemcpyDefault, d->stream),
              "write slots");
        check(cudaStreamSynchronize(d->stream), "write");
    });
}

void chroma_b200_decoder_destroy(chroma_b200_decoder* d) { delete d; }

int chroma_b200_host_alloc(size_t bytes, void** out, char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!out) throw ValueError("null argument");
        *out = nullptr;
        check(cudaMallocHost(out, bytes ? bytes : 1), "cudaMallocHost");
    });
}

void chroma_b200_host_free(void* p) {
    if (p) cudaFreeHost(p);
}

}  // extern "C"
