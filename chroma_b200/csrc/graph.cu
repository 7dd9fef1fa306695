// Generic exported graphs: any graph over the reference's operator table (chroma/_src/lowering.py:34-86) that is
// not one of the recognised GPT-OSS programs, run by a handful of precompiled kernels driven by a launch plan.
//
// The reference generates one C++/CUDA kernel per fused expression and builds it with nvcc per graph
// (chroma/_src/codegen/gpu.py:63-435, chroma/_src/codegen/cuda/codegen.py:44-168). Here the compiler
// (chroma_b200/_src/graph.py) lowers the graph to a plan of steps over strided views of the program's buffers
// (inputs, outputs, one arena, the weights), and these kernels interpret it:
//
//   kGElementwise  a fused elementwise expression per output element: a register bytecode over strided, broadcast
//                  operand views (loads, + - * / with IEEE rounding and no contraction, the unary functions of the
//                  reference's table, pow, clamp, bf16 rounding after every op of a bf16 result), stored to a view
//   kGMove         element copy between views of the same type (int64 included), optionally keeping only the upper
//                  or lower triangle (triu / tril, kernels.h:117-123) -- views, concatenation parts, outputs
//   kGReduce       sum / mean over axes: a sequential fp32 sum over the reduced index space, divided by the count
//   kGContract     linear and einsum: per output element a sequential fp32 sum of products over the contracted
//                  index space (the portable gemm / loop einsum of kernels.h:24-74), + bias
//   kGSoftmax      the three passes of kernels.h:125-151 along an axis
//   kGTopk         top-k along an axis: NaN ranks highest (largest) or last (smallest), ties to the lowest index,
//                  sorted (the ranking of chroma/_src/codegen/gpu.py:300-311)
//   kGGather       embedding / index rows with the reference's bounds check (negative rows wrap for aten.index)
//
// One thread per output element (or row), grid-stride; the arithmetic uses the round-to-nearest intrinsics so the
// compiler cannot fuse a multiply into an add, which keeps sums and products bit-identical to the reference's
// portable CPU build (-ffp-contract=off, chroma/_src/build.py:19); exp/sin/cos/pow follow CUDA's libm.
#include "../../include/chroma_b200.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

constexpr int kGMaxRank = 8;
constexpr int kGMaxRegs = 32;
constexpr unsigned kGErrIndex = 1u;

enum GKind : int { kGElementwise = 1, kGMove, kGReduce, kGContract, kGSoftmax, kGTopk, kGGather };
enum GType : int { kF32 = 0, kBF16 = 1, kI64 = 2 };
enum GOpCode : int {
    kOpLoad = 1, kOpConst, kOpAdd, kOpSub, kOpMul, kOpDiv, kOpNeg, kOpAbs, kOpExp, kOpSin, kOpCos, kOpRecip,
    kOpRsqrt, kOpSigmoid, kOpSquare, kOpPow, kOpMaxC, kOpMinC, kOpRound
};

struct GView {
    char* ptr;  // first element (offset applied)
    int dtype, rank;
    long long shape[kGMaxRank], stride[kGMaxRank];  // in elements
};

struct GOp {
    int op, dst, a, b;
    float imm;
};

struct GStep {
    int kind, rank;                   // iteration rank (the output's)
    long long n;                      // work items: output elements, or rows for softmax / top-k
    long long oshape[kGMaxRank];      // iteration shape
    int out, out2, in, in2, bias;     // view indices (-1: none)
    int first_operand, n_operands, first_op, n_ops;
    int rrank;                        // reduction rank (reduce / contract)
    long long rshape[kGMaxRank], rstride_a[kGMaxRank], rstride_b[kGMaxRank];
    int axis, k, largest, tri, diag, negative;  // softmax / top-k axis (of the iteration shape) ...
    long long width;                  // ... its length; top-k k; triangle mode (0, 1 upper, 2 lower)
    float divisor;
};

__device__ __forceinline__ int es_of(int t) { return t == kI64 ? 8 : (t == kBF16 ? 2 : 4); }

__device__ __forceinline__ float load_f(const GView& v, long long off) {
    if (v.dtype == kBF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(v.ptr)[off]);
    return reinterpret_cast<const float*>(v.ptr)[off];
}
__device__ __forceinline__ void store_f(const GView& v, long long off, float x) {
    if (v.dtype == kBF16) reinterpret_cast<__nv_bfloat16*>(v.ptr)[off] = __float2bfloat16_rn(x);
    else reinterpret_cast<float*>(v.ptr)[off] = x;
}
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Coordinates of linear index i in `shape` (row-major).
__device__ __forceinline__ void coords(long long i, int rank, const long long* shape, long long* c) {
    for (int d = rank - 1; d >= 0; --d) {
        c[d] = i % shape[d];
        i /= shape[d];
    }
}
__device__ __forceinline__ long long offset_of(const GView& v, int rank, const long long* c) {
    long long o = 0;
    for (int d = 0; d < rank; ++d) o += c[d] * v.stride[d];
    return o;
}

__global__ void k_g_elementwise(const GStep* steps, int s, const GView* views, const GOp* ops) {
    const GStep& st = steps[s];
    const GView& out = views[st.out];
    float r[kGMaxRegs];
    long long c[kGMaxRank];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        int last = 0;
        for (int j = 0; j < st.n_ops; ++j) {
            const GOp o = ops[st.first_op + j];
            float v;
            switch (o.op) {
                case kOpLoad: {
                    const GView& x = views[st.first_operand + o.a];
                    v = load_f(x, offset_of(x, st.rank, c));
                    break;
                }
                case kOpConst: v = o.imm; break;
                case kOpAdd: v = __fadd_rn(r[o.a], r[o.b]); break;
                case kOpSub: v = __fsub_rn(r[o.a], r[o.b]); break;
                case kOpMul: v = __fmul_rn(r[o.a], r[o.b]); break;
                case kOpDiv: v = __fdiv_rn(r[o.a], r[o.b]); break;
                case kOpNeg: v = -r[o.a]; break;
                case kOpAbs: v = fabsf(r[o.a]); break;
                case kOpExp: v = expf(r[o.a]); break;
                case kOpSin: v = sinf(r[o.a]); break;
                case kOpCos: v = cosf(r[o.a]); break;
                case kOpRecip: v = __fdiv_rn(1.0f, r[o.a]); break;
                case kOpRsqrt: v = __fdiv_rn(1.0f, __fsqrt_rn(r[o.a])); break;
                case kOpSigmoid: v = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-r[o.a]))); break;
                case kOpSquare: v = __fmul_rn(r[o.a], r[o.a]); break;
                case kOpPow: v = powf(r[o.a], r[o.b]); break;
                case kOpMaxC: v = (r[o.a] < o.imm) ? o.imm : r[o.a]; break;  // std::max(x, low): NaN stays
                case kOpMinC: v = (o.imm < r[o.a]) ? o.imm : r[o.a]; break;  // std::min(x, high): NaN stays
                case kOpRound: v = round_bf16(r[o.a]); break;
                default: v = 0.f; break;
            }
            r[o.dst] = v;
            last = o.dst;
        }
        store_f(out, offset_of(out, st.rank, c), r[last]);
    }
}

__global__ void k_g_move(const GStep* steps, int s, const GView* views) {
    const GStep& st = steps[s];
    const GView& out = views[st.out];
    const GView& in = views[st.in];
    const int es = es_of(out.dtype);
    long long c[kGMaxRank];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        bool keep = true;
        if (st.tri) {
            const long long diag = c[st.rank - 1] - c[st.rank - 2];
            keep = st.tri == 1 ? diag >= st.diag : diag <= st.diag;
        }
        char* dst = out.ptr + offset_of(out, st.rank, c) * es;
        const char* src = in.ptr + offset_of(in, st.rank, c) * es;
        if (es == 8) *reinterpret_cast<long long*>(dst) = keep ? *reinterpret_cast<const long long*>(src) : 0ll;
        else if (es == 4) *reinterpret_cast<unsigned*>(dst) = keep ? *reinterpret_cast<const unsigned*>(src) : 0u;
        else *reinterpret_cast<unsigned short*>(dst) = keep ? *reinterpret_cast<const unsigned short*>(src) : 0;
    }
}

// Sum over the reduced index space (row-major, sequential), then / divisor (1 for sum, the count for mean).
__global__ void k_g_reduce(const GStep* steps, int s, const GView* views) {
    const GStep& st = steps[s];
    const GView& out = views[st.out];
    const GView& in = views[st.in];
    long long c[kGMaxRank], rc[kGMaxRank];
    long long rn = 1;
    for (int d = 0; d < st.rrank; ++d) rn *= st.rshape[d];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        const long long base = offset_of(in, st.rank, c);
        float sum = 0.f;
        for (long long j = 0; j < rn; ++j) {
            coords(j, st.rrank, st.rshape, rc);
            long long o = base;
            for (int d = 0; d < st.rrank; ++d) o += rc[d] * st.rstride_a[d];
            sum = __fadd_rn(sum, load_f(in, o));
        }
        store_f(out, offset_of(out, st.rank, c), __fdiv_rn(sum, st.divisor));
    }
}

// out = sum over the contracted index space of a * b (+ bias): linear (x . W^T + b) and einsum.
__global__ void k_g_contract(const GStep* steps, int s, const GView* views) {
    const GStep& st = steps[s];
    const GView& out = views[st.out];
    const GView& a = views[st.in];
    const GView& b = views[st.in2];
    long long c[kGMaxRank], rc[kGMaxRank];
    long long rn = 1;
    for (int d = 0; d < st.rrank; ++d) rn *= st.rshape[d];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        const long long ba = offset_of(a, st.rank, c), bb = offset_of(b, st.rank, c);
        float sum = 0.f;
        for (long long j = 0; j < rn; ++j) {
            coords(j, st.rrank, st.rshape, rc);
            long long oa = ba, ob = bb;
            for (int d = 0; d < st.rrank; ++d) {
                oa += rc[d] * st.rstride_a[d];
                ob += rc[d] * st.rstride_b[d];
            }
            sum = __fadd_rn(sum, __fmul_rn(load_f(a, oa), load_f(b, ob)));
        }
        if (st.bias >= 0) {
            const GView& bv = views[st.bias];
            sum = __fadd_rn(sum, load_f(bv, offset_of(bv, st.rank, c)));
        }
        store_f(out, offset_of(out, st.rank, c), sum);
    }
}

// One thread per row along `axis` (iteration shape has that axis at extent 1).
__global__ void k_g_softmax(const GStep* steps, int s, const GView* views) {
    const GStep& st = steps[s];
    const GView& out = views[st.out];
    const GView& in = views[st.in];
    long long c[kGMaxRank];
    const long long si = in.stride[st.axis], so = out.stride[st.axis];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        const long long bi = offset_of(in, st.rank, c), bo = offset_of(out, st.rank, c);
        float m = -INFINITY;
        for (long long k = 0; k < st.width; ++k) {
            const float v = load_f(in, bi + k * si);
            m = (m < v) ? v : m;  // std::max(maximum, v)
        }
        float sum = 0.f;
        for (long long k = 0; k < st.width; ++k) sum = __fadd_rn(sum, expf(__fsub_rn(load_f(in, bi + k * si), m)));
        for (long long k = 0; k < st.width; ++k)
            store_f(out, bo + k * so, __fdiv_rn(expf(__fsub_rn(load_f(in, bi + k * si), m)), sum));
    }
}

// a ranks before b (largest: NaN first, then larger; smallest: numbers before NaN, then smaller); ties: lower index.
__device__ __forceinline__ bool ranks_before(float a, long long ia, float b, long long ib, bool largest) {
    const bool na = isnan(a), nb = isnan(b);
    if (largest) {
        if (na != nb) return na;
        if (!na && a != b) return a > b;
    } else {
        if (na != nb) return nb;
        if (!na && a != b) return a < b;
    }
    return ia < ib;
}

__global__ void k_g_topk(const GStep* steps, int s, const GView* views) {
    const GStep& st = steps[s];
    const GView& vo = views[st.out];
    const GView& io = views[st.out2];
    const GView& in = views[st.in];
    long long c[kGMaxRank];
    const long long si = in.stride[st.axis], sv = vo.stride[st.axis], sx = io.stride[st.axis];
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        const long long bi = offset_of(in, st.rank, c), bv = offset_of(vo, st.rank, c), bx = offset_of(io, st.rank, c);
        // Selection by rank: the j-th output is the element with exactly j elements ranked before it.
        float prev = 0.f;
        long long prev_i = -1;
        for (int j = 0; j < st.k; ++j) {
            float best = 0.f;
            long long best_i = -1;
            for (long long q = 0; q < st.width; ++q) {
                const float v = load_f(in, bi + q * si);
                if (prev_i >= 0 && !ranks_before(prev, prev_i, v, q, st.largest)) continue;  // already taken
                if (best_i < 0 || ranks_before(v, q, best, best_i, st.largest)) {
                    best = v;
                    best_i = q;
                }
            }
            store_f(vo, bv + j * sv, best);
            reinterpret_cast<long long*>(io.ptr)[bx + j * sx] = best_i;
            prev = best;
            prev_i = best_i;
        }
    }
}

// out[i0.., rest..] = table[idx[i0..], rest..]; rows outside [0, rows) (after wrapping negatives for aten.index)
// raise the index error and write zeros.
__global__ void k_g_gather(const GStep* steps, int s, const GView* views, unsigned* err) {
    const GStep& st = steps[s];
    const GView& out = views[st.out];
    const GView& tab = views[st.in];
    const GView& idx = views[st.in2];
    const int es = es_of(out.dtype);
    long long c[kGMaxRank], tc[kGMaxRank];
    const int ir = idx.rank, tr = tab.rank;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < st.n; i += (long long)gridDim.x * blockDim.x) {
        coords(i, st.rank, st.oshape, c);
        long long row = reinterpret_cast<const long long*>(idx.ptr)[offset_of(idx, ir, c)];
        const long long rows = tab.shape[0];
        if (st.negative && row < 0) row += rows;
        char* dst = out.ptr + offset_of(out, st.rank, c) * es;
        if (row < 0 || row >= rows) {
            atomicOr(err, kGErrIndex);
            memset(dst, 0, es);
            continue;
        }
        tc[0] = row;
        for (int d = 1; d < tr; ++d) tc[d] = c[ir + d - 1];
        const char* src = tab.ptr + offset_of(tab, tr, tc) * es;
        memcpy(dst, src, es);
    }
}

// ---------------------------------------------------------------------------------------------------------
struct DeviceGuard {
    int prev = 0;
    explicit DeviceGuard(int device) {
        cudaGetDevice(&prev);
        cudaSetDevice(device);
    }
    ~DeviceGuard() { cudaSetDevice(prev); }
};

struct ValueError : std::runtime_error {
    using std::runtime_error::runtime_error;
};
struct IndexError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

struct DevMem {
    void* p = nullptr;
    size_t bytes = 0;
    DevMem() = default;
    explicit DevMem(size_t n) : bytes(n) {
        if (n) check(cudaMalloc(&p, n), "cudaMalloc");
    }
    DevMem(const DevMem&) = delete;
    DevMem& operator=(const DevMem&) = delete;
    DevMem(DevMem&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
    DevMem& operator=(DevMem&& o) noexcept {
        std::swap(p, o.p);
        std::swap(bytes, o.bytes);
        return *this;
    }
    ~DevMem() {
        if (p) cudaFree(p);
    }
};

// Plan words (int64, little endian): see chroma_b200/_src/graph.py `Plan.words`.
constexpr long long kMagic = 0x31474243;  // "CBG1"

struct Reader {
    const int64_t* w;
    size_t n, i = 0;
    long long next() {
        if (i >= n) throw ValueError("truncated graph plan");
        return w[i++];
    }
};

}  // namespace

struct chroma_b200_graph {
    int device = 0;
    std::string name;
    cudaStream_t stream = nullptr;
    DevMem weights, arena, err, d_views, d_ops, d_steps;
    std::vector<DevMem> in_bufs, out_bufs;
    std::vector<size_t> in_bytes, out_bytes;
    std::vector<GStep> steps;
    std::vector<int> grids;
    unsigned* err_host = nullptr;
    int sms = 148;

    ~chroma_b200_graph() {
        DeviceGuard g(device);
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        if (err_host) cudaFreeHost(err_host);
    }
};

namespace {

int fail(char* err, size_t n, int code, const char* msg) {
    if (err && n) {
        std::strncpy(err, msg, n - 1);
        err[n - 1] = '\0';
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
    }
}

void build(chroma_b200_graph& g, const int64_t* words, size_t count, const char* weights_path) {
    Reader r{words, count};
    if (r.next() != kMagic) throw ValueError("not a chroma_b200 graph plan");
    const long long weight_bytes = r.next(), arena_bytes = r.next();
    const long long n_in = r.next(), n_out = r.next();
    if (weight_bytes < 0 || arena_bytes < 0 || n_in < 0 || n_out < 1 || n_in > 4096 || n_out > 4096)
        throw ValueError("graph plan header out of range");
    for (long long i = 0; i < n_in; ++i) g.in_bytes.push_back(size_t(r.next()));
    for (long long i = 0; i < n_out; ++i) g.out_bytes.push_back(size_t(r.next()));
    // Device buffers.
    g.weights = DevMem(size_t(weight_bytes));
    if (weight_bytes) {
        if (!weights_path) throw ValueError("graph plan needs weights");
        FILE* f = std::fopen(weights_path, "rb");
        if (!f) throw std::runtime_error("Missing weights file or incorrect byte size");
        std::vector<char> host(size_t(weight_bytes) + 1);
        const size_t got = std::fread(host.data(), 1, host.size(), f);
        std::fclose(f);
        if (got != size_t(weight_bytes)) throw std::runtime_error("Missing weights file or incorrect byte size");
        check(cudaMemcpy(g.weights.p, host.data(), size_t(weight_bytes), cudaMemcpyHostToDevice), "weights upload");
    }
    g.arena = DevMem(size_t(arena_bytes));
    for (size_t b : g.in_bytes) g.in_bufs.emplace_back(b);
    for (size_t b : g.out_bytes) g.out_bufs.emplace_back(b);
    auto base = [&](long long kind, long long index, long long bytes) -> char* {
        // kind 0: input `index`; 1: output `index`; 2: arena at byte `index`; 3: weights at byte `index`.
        if (kind == 0 && index >= 0 && index < n_in) {
            if (bytes > (long long)g.in_bytes[size_t(index)]) throw ValueError("view past an input");
            return static_cast<char*>(g.in_bufs[size_t(index)].p);
        }
        if (kind == 1 && index >= 0 && index < n_out) {
            if (bytes > (long long)g.out_bytes[size_t(index)]) throw ValueError("view past an output");
            return static_cast<char*>(g.out_bufs[size_t(index)].p);
        }
        if (kind == 2 && index >= 0 && index + bytes <= arena_bytes) return static_cast<char*>(g.arena.p) + index;
        if (kind == 3 && index >= 0 && index + bytes <= weight_bytes) return static_cast<char*>(g.weights.p) + index;
        throw ValueError("graph plan view outside its buffer");
    };
    // Views.
    const long long n_views = r.next();
    if (n_views < 0 || n_views > (1 << 20)) throw ValueError("graph plan view count out of range");
    std::vector<GView> views(static_cast<size_t>(n_views));
    for (auto& v : views) {
        const long long kind = r.next(), index = r.next(), span = r.next();
        v.dtype = int(r.next());
        v.rank = int(r.next());
        const long long offset = r.next();
        if (v.rank < 0 || v.rank > kGMaxRank || v.dtype < kF32 || v.dtype > kI64) throw ValueError("bad graph view");
        const int es = v.dtype == kI64 ? 8 : (v.dtype == kBF16 ? 2 : 4);
        // `span` = elements from the view's first to one past its last element (checked on the host side of the
        // plan); the buffer must hold the offset plus that span.
        v.ptr = base(kind, index, (offset + span) * es) + offset * es;
        for (int d = 0; d < kGMaxRank; ++d) {
            v.shape[d] = r.next();
            v.stride[d] = r.next();
        }
    }
    // Ops.
    const long long n_ops = r.next();
    if (n_ops < 0 || n_ops > (1 << 22)) throw ValueError("graph plan op count out of range");
    std::vector<GOp> ops(static_cast<size_t>(n_ops));
    for (auto& o : ops) {
        const long long a = r.next(), imm = r.next();
        o.op = int(a & 0xff);
        o.dst = int((a >> 8) & 0xff);
        o.a = int((a >> 16) & 0xff);
        o.b = int((a >> 24) & 0xff);
        const uint32_t bits = uint32_t(imm);
        std::memcpy(&o.imm, &bits, 4);
        if (o.dst >= kGMaxRegs || o.a >= kGMaxRegs || o.b >= kGMaxRegs) throw ValueError("graph op register out of range");
    }
    // Steps.
    const long long n_steps = r.next();
    if (n_steps < 0 || n_steps > (1 << 20)) throw ValueError("graph plan step count out of range");
    auto view_index = [&](long long v, bool optional) -> int {
        if (optional && v < 0) return -1;
        if (v < 0 || v >= n_views) throw ValueError("graph step names a missing view");
        return int(v);
    };
    for (long long sidx = 0; sidx < n_steps; ++sidx) {
        GStep st{};
        st.kind = int(r.next());
        st.rank = int(r.next());
        st.n = r.next();
        if (st.rank < 0 || st.rank > kGMaxRank || st.n < 0) throw ValueError("bad graph step");
        for (int d = 0; d < kGMaxRank; ++d) st.oshape[d] = r.next();
        st.out = view_index(r.next(), false);
        st.out2 = view_index(r.next(), true);
        st.in = view_index(r.next(), true);
        st.in2 = view_index(r.next(), true);
        st.bias = view_index(r.next(), true);
        st.first_operand = int(r.next());
        st.n_operands = int(r.next());
        st.first_op = int(r.next());
        st.n_ops = int(r.next());
        st.rrank = int(r.next());
        if (st.rrank < 0 || st.rrank > kGMaxRank) throw ValueError("bad graph reduction rank");
        for (int d = 0; d < kGMaxRank; ++d) {
            st.rshape[d] = r.next();
            st.rstride_a[d] = r.next();
            st.rstride_b[d] = r.next();
        }
        st.axis = int(r.next());
        st.width = r.next();
        st.k = int(r.next());
        st.largest = int(r.next());
        st.tri = int(r.next());
        st.diag = int(r.next());
        st.negative = int(r.next());
        const uint32_t dbits = uint32_t(r.next());
        std::memcpy(&st.divisor, &dbits, 4);
        if (st.first_operand < 0 || st.n_operands < 0 || st.first_operand + st.n_operands > n_views ||
            st.first_op < 0 || st.n_ops < 0 || st.first_op + st.n_ops > n_ops)
            throw ValueError("graph step names missing operands or ops");
        if (st.kind < kGElementwise || st.kind > kGGather) throw ValueError("unknown graph step kind");
        if ((st.kind == kGContract || st.kind == kGGather) && st.in2 < 0) throw ValueError("graph step lacks an operand");
        if (st.kind != kGElementwise && st.in < 0) throw ValueError("graph step lacks its input");
        if (st.kind == kGTopk && st.out2 < 0) throw ValueError("top-k step lacks its index output");
        if ((st.kind == kGSoftmax || st.kind == kGTopk) && (st.axis < 0 || st.axis >= st.rank)) throw ValueError("bad axis");
        g.steps.push_back(st);
        const long long blocks = (st.n + 255) / 256;
        g.grids.push_back(int(blocks < 1 ? 1 : (blocks > 8 * g.sms ? 8 * g.sms : blocks)));
    }
    if (r.i != r.n) throw ValueError("trailing words in the graph plan");
    g.d_views = DevMem(views.size() * sizeof(GView));
    g.d_ops = DevMem(ops.size() * sizeof(GOp));
    g.d_steps = DevMem(g.steps.size() * sizeof(GStep));
    if (!views.empty()) check(cudaMemcpy(g.d_views.p, views.data(), g.d_views.bytes, cudaMemcpyHostToDevice), "views");
    if (!ops.empty()) check(cudaMemcpy(g.d_ops.p, ops.data(), g.d_ops.bytes, cudaMemcpyHostToDevice), "ops");
    if (!g.steps.empty()) check(cudaMemcpy(g.d_steps.p, g.steps.data(), g.d_steps.bytes, cudaMemcpyHostToDevice), "steps");
}

void enqueue(chroma_b200_graph& g) {
    const GStep* steps = static_cast<const GStep*>(g.d_steps.p);
    const GView* views = static_cast<const GView*>(g.d_views.p);
    const GOp* ops = static_cast<const GOp*>(g.d_ops.p);
    unsigned* err = static_cast<unsigned*>(g.err.p);
    for (size_t s = 0; s < g.steps.size(); ++s) {
        const dim3 grid(unsigned(g.grids[s])), block(256);
        const int si = int(s);
        switch (g.steps[s].kind) {
            case kGElementwise: k_g_elementwise<<<grid, block, 0, g.stream>>>(steps, si, views, ops); break;
            case kGMove: k_g_move<<<grid, block, 0, g.stream>>>(steps, si, views); break;
            case kGReduce: k_g_reduce<<<grid, block, 0, g.stream>>>(steps, si, views); break;
            case kGContract: k_g_contract<<<grid, block, 0, g.stream>>>(steps, si, views); break;
            case kGSoftmax: k_g_softmax<<<grid, block, 0, g.stream>>>(steps, si, views); break;
            case kGTopk: k_g_topk<<<grid, block, 0, g.stream>>>(steps, si, views); break;
            case kGGather: k_g_gather<<<grid, block, 0, g.stream>>>(steps, si, views, err); break;
            default: break;
        }
    }
    check(cudaGetLastError(), "graph launch");
}

}  // namespace

extern "C" {

int chroma_b200_graph_create(const int64_t* plan, size_t words, const char* weights_path, chroma_b200_graph** out,
                             char* err, size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!plan || !out) throw ValueError("null argument");
        auto g = std::make_unique<chroma_b200_graph>();
        check(cudaGetDevice(&g->device), "cudaGetDevice");
        cudaDeviceProp prop{};
        check(cudaGetDeviceProperties(&prop, g->device), "cudaGetDeviceProperties");
        if (prop.major != 10)
            throw std::runtime_error(std::string("chroma_b200 kernels are built for sm_100a (B200); found ") + prop.name);
        g->name = prop.name;
        g->sms = prop.multiProcessorCount;
        check(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking), "cudaStreamCreateWithFlags");
        g->err = DevMem(sizeof(unsigned));
        check(cudaMemset(g->err.p, 0, sizeof(unsigned)), "error word");
        check(cudaMallocHost(reinterpret_cast<void**>(&g->err_host), sizeof(unsigned)), "cudaMallocHost");
        build(*g, plan, words, weights_path);
        *out = g.release();
    });
}

int chroma_b200_graph_run(chroma_b200_graph* g, const void* const* inputs, void* const* outputs, char* err,
                          size_t err_len) {
    return guarded(err, err_len, [&] {
        if (!g || (!inputs && !g->in_bufs.empty()) || !outputs) throw ValueError("null argument");
        DeviceGuard guard(g->device);
        for (size_t i = 0; i < g->in_bufs.size(); ++i)
            check(cudaMemcpyAsync(g->in_bufs[i].p, inputs[i], g->in_bytes[i], cudaMemcpyHostToDevice, g->stream),
                  "input upload");
        enqueue(*g);
        check(cudaMemcpyAsync(g->err_host, g->err.p, sizeof(unsigned), cudaMemcpyDeviceToHost, g->stream), "error word");
        check(cudaMemsetAsync(g->err.p, 0, sizeof(unsigned), g->stream), "error word");
        for (size_t i = 0; i < g->out_bufs.size(); ++i)
            check(cudaMemcpyAsync(outputs[i], g->out_bufs[i].p, g->out_bytes[i], cudaMemcpyDeviceToHost, g->stream),
                  "output download");
        // Synchronise before reporting anything: the host buffers must outlive the copies (runtime.h:168-172).
        check(cudaStreamSynchronize(g->stream), "CUDA execution");
        if (*g->err_host & kGErrIndex) throw IndexError("Tensor idx out of range");
    });
}

const char* chroma_b200_graph_device(const chroma_b200_graph* g) { return g ? g->name.c_str() : ""; }

int32_t chroma_b200_graph_launches(const chroma_b200_graph* g) { return g ? int32_t(g->steps.size()) : 0; }

void chroma_b200_graph_destroy(chroma_b200_graph* g) { delete g; }

}  // extern "C"
