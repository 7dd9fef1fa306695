/* chroma_b200: C ABI of the B200-native (sm_100a) backend for Chroma's compiled GPT-OSS-style programs.
 *
 * Every entry point takes plain pointers and sizes. Host buffers are caller-owned; all device memory is owned
 * by the objects created here. Calls return a status code; on failure a NUL-terminated message is written to
 * `err` (at most `err_len` bytes, may be NULL).
 *
 * The boundary replaces the native side of a compiled reference artefact:
 *   - `create_model(const char* weights_file)` and `ModelProgram::run(const void* const* inputs,
 *     void* const* outputs)` emitted by the CUDA generator (chroma/_src/codegen/cuda/codegen.py:13-41), and
 *   - the runtime they drive, `chroma::cuda::Runner::{initialize, run}` (chroma/_src/codegen/cuda/runtime.h:116-173),
 *   - exposed to Python as `Model(weights).run(inputs, outputs)` / `.device` (chroma/_src/core/bindings.h:35-75).
 */
#ifndef CHROMA_B200_H
#define CHROMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. They map to the exceptions the reference raises (runtime.h:63-73 and :160-162,
 * bindings.h:17-33): INDEX -> IndexError, VALUE -> ValueError, RUNTIME -> RuntimeError. */
#define CHROMA_B200_OK 0
#define CHROMA_B200_INDEX 1
#define CHROMA_B200_VALUE 2
#define CHROMA_B200_RUNTIME 3

/* Program kinds (what one `run` computes). */
#define CHROMA_B200_GPTOSS_FORWARD 1 /* Transformer.forward: tokens[n] -> logits[n, V] (gpt_oss.py:304-310) */
#define CHROMA_B200_GPTOSS_CACHED 2  /* CachedTransformer step: 7 inputs -> 3 outputs (cached.py:16-51) */
#define CHROMA_B200_MICRO 3          /* rmsnorm(x)*w -> z=y*g -> z*sigmoid(z)*u + x, bf16 [rows, cols] */
#define CHROMA_B200_GPTOSS_LAST 4    /* UncachedTransformer: tokens[n], position[1] -> logits[1, V] (cached.py:54-65) */

#define CHROMA_B200_FP32 0
#define CHROMA_B200_BF16 1

/* Weight tensors of a GPT-OSS program, as byte offsets into the weights file, in this order:
 *   [0] embedding [V, d]       [1] final norm scale [d] (fp32)   [2] unembedding [V, d]
 *   then per layer l, at 3 + 13*l + i:
 *   i=0 attn norm [d] (fp32)   1 sinks [H]   2 qkv.weight [(H+2KV)*hd, d]   3 qkv.bias   4 out.weight [d, H*hd]
 *   5 out.bias [d]   6 mlp norm [d] (fp32)   7 gate.weight [E, d]   8 gate.bias [E]   9 mlp1_weight [E, 2I, d]
 *   10 mlp1_bias [E, 2I]   11 mlp2_weight [E, d, I]   12 mlp2_bias [E, d]
 * Tensors other than the norm scales are in the program's storage type. Offsets are 256-byte aligned.
 * A MICRO program has a single tensor: [0] the fp32 norm weight [cols]. */
typedef struct chroma_b200_desc {
    int32_t kind;
    int32_t storage;
    int32_t layers, hidden, heads, kv_heads, head_dim, experts, top_k, intermediate, vocab;
    int32_t tokens;      /* rows per call (n) */
    int32_t context;     /* cache rows (CACHED) */
    int32_t window;      /* sliding window of the layers that use one (0 = none) */
    float eps, sm_scale, swiglu_alpha, swiglu_limit, rope_concentration;
    int64_t rows, cols;  /* MICRO shape */
    const float* inv_freq;        /* [head_dim / 2] RoPE inverse frequencies */
    const int32_t* layer_window;  /* [layers]: 1 if the layer uses the window (mask) input */
    const int64_t* offsets;       /* weight offsets, see above */
    int32_t num_offsets;
    int64_t weight_bytes;         /* exact size of the weights file */
} chroma_b200_desc;

typedef struct chroma_b200_program chroma_b200_program;
typedef struct chroma_b200_decoder chroma_b200_decoder;

/* Loads the weights once and allocates every device buffer a call needs on the CURRENT device
 * (the reference binds a Program to the current device the same way, runtime.h:118).
 * Replaces create_model()/Runner::initialize. */
int chroma_b200_create(const chroma_b200_desc* desc, const char* weights_path, chroma_b200_program** out,
                       char* err, size_t err_len);

/* Same as chroma_b200_create, with the weights already in device memory of the current device, laid out as the
 * weights file would be (`desc->offsets`). They are not copied: the caller keeps them alive until destroy. For
 * weights generated on the device (benchmarks) or shared with another runtime. No reference counterpart. */
int chroma_b200_create_device(const chroma_b200_desc* desc, const void* device_weights, chroma_b200_program** out,
                              char* err, size_t err_len);

/* One call on host buffers: uploads inputs, runs, downloads outputs, synchronises. Input and output
 * order and byte sizes are those of the program's manifest. Replaces ModelProgram::run / Runner::run. */
int chroma_b200_run(chroma_b200_program* program, const void* const* inputs, void* const* outputs, char* err,
                    size_t err_len);

/* Device-resident execution for benchmarks and fused pipelines: device pointers of the program's own input
 * and output buffers (valid until destroy), and one run on them, queued on `stream` (a cudaStream_t, 0 for the
 * program's own stream). `chroma_b200_run_device` does not synchronise; it returns after queuing. */
int chroma_b200_buffers(chroma_b200_program* program, void** inputs, void** outputs, char* err, size_t err_len);
int chroma_b200_run_device(chroma_b200_program* program, void* stream, char* err, size_t err_len);
/* Reads and clears the program's device error word after a run_device (synchronises `stream`). */
int chroma_b200_check(chroma_b200_program* program, void* stream, char* err, size_t err_len);

/* Device name of the program's GPU (bindings.h:39 `device`). */
const char* chroma_b200_device(const chroma_b200_program* program);
/* Number of kernels one run launches (for launch accounting). */
int32_t chroma_b200_launches(const chroma_b200_program* program);
void chroma_b200_destroy(chroma_b200_program* program);

/* Activation arena planner used by every program: best fit over inclusive [start, end] kernel-index lifetimes with
 * a coalesced free list, visiting allocations by start (the reference's plan_memory, chroma/_src/memory.py:12-50).
 * Writes each allocation's byte offset and returns the arena size (-1 on bad arguments). Needs no GPU. */
int64_t chroma_b200_plan_arena(int32_t count, const int64_t* sizes, const int32_t* starts, const int32_t* ends,
                               int64_t* offsets);
/* Routing of the last run of a GPT-OSS program: the selected experts [layers, tokens, top_k] in rank order (the
 * indices of torch.topk(..., sorted=True) at gpt_oss.py:246), for parity checks. `count` is the element count. */
int chroma_b200_routes(chroma_b200_program* program, int32_t* out, int64_t count, char* err, size_t err_len);
/* Vocab projection with greedy argmax that allocates nothing (no counterpart in the reference). For callers that
 * cannot call cudaMalloc, such as code running inside another framework's stream capture or an allocator-free host:
 * `x` [rows, hidden] fp32 final-normed rows and `ids` [rows] int64 (and `logits` [rows, vocab] in the program's
 * storage type, or NULL) are caller-owned device buffers; the program supplies the unembedding weights it already
 * holds. Scratch is a static device array of 256 rows (2 KiB) held by every GPU that loads the library: rows > 256
 * is a CHROMA_B200_VALUE error. The first call on a device looks up that array's device address, so make it before
 * any stream capture. Calls share the array: calls that overlap on the GPU race. A vocab-sharded expert-parallel
 * program (it holds only its rank's unembedding rows) is a CHROMA_B200_VALUE error. Queued on `stream` (a
 * cudaStream_t; 0 is the legacy default stream), not synchronised. */
int chroma_b200_vocab_argmax_static(const chroma_b200_program* program, const float* x, int32_t rows, void* logits,
                                    int64_t* ids, void* stream, char* err, size_t err_len);
/* ---- Generic exported graphs -------------------------------------------------------------------------------------
 * Graphs over the reference's operator table (chroma/_src/lowering.py:34-86) other than the recognised GPT-OSS
 * programs. Replaces the per-graph generated kernels and their build (chroma/_src/codegen/gpu.py:63-435,
 * chroma/_src/codegen/cuda/codegen.py:44-168, chroma/_src/build.py:22-30) with precompiled kernels driven by a plan:
 * `plan` is `words` int64 values written by chroma_b200/_src/graph.py (buffers, strided views, elementwise bytecode,
 * steps); `weights_path` holds the graph's parameters and folded constants (NULL when it has none). Created on the
 * current device. `run` has the contract of chroma_b200_run (host buffers in manifest order, synchronises; an index
 * out of range is CHROMA_B200_INDEX with the program still usable, as Runner::run, runtime.h:147-173). */
typedef struct chroma_b200_graph chroma_b200_graph;
int chroma_b200_graph_create(const int64_t* plan, size_t words, const char* weights_path, chroma_b200_graph** out,
                             char* err, size_t err_len);
int chroma_b200_graph_run(chroma_b200_graph* graph, const void* const* inputs, void* const* outputs, char* err,
                          size_t err_len);
const char* chroma_b200_graph_device(const chroma_b200_graph* graph);
int32_t chroma_b200_graph_launches(const chroma_b200_graph* graph);
void chroma_b200_graph_destroy(chroma_b200_graph* graph);

/* GEMM epilogues of chroma_b200_gemm_bf16. */
#define CHROMA_B200_EPI_STORE 0    /* C = bf16(A.B^T + bias) (nn.Linear, chroma/_src/codegen/cpu/kernels.h:63-74) */
#define CHROMA_B200_EPI_RESIDUAL 1 /* C = bf16(R + bf16(A.B^T + bias)): linear + residual (gpt_oss.py:209) */
#define CHROMA_B200_EPI_SWIGLU 2   /* C[:, p] = SwiGLU of column pair (2p, 2p+1) (gpt_oss.py:212-219, 253-254) */
#define CHROMA_B200_EPI_EXPERT 3   /* C = bf16(bf16(A.B^T) + bias[group]): expert einsum + bias (gpt_oss.py:259-260) */

/* bf16 tensor-core GEMM on device buffers, C = A[m, k] . B^T with B stored [groups * n, k] row-major (nn.Linear
 * layout), fp32 accumulation, fused epilogue. Dense when `offsets` is NULL (groups = 1). Grouped (MoE experts) when
 * `offsets` [groups + 1] (device, int32) gives each group's row range in A: rows of group g use B rows
 * [g*n, (g+1)*n) and bias row g. `tile_scratch` is unused (kept for binary compatibility; may be NULL). C has n columns
 * (n / 2 for the SwiGLU epilogue). Replaces the cuBLAS SGEMM of Runner::linear (runtime.h:175-181) and the generated
 * per-expert einsum loops (gpu.py:390-424). Queued on `stream`; a stuck pipeline sets bit 2 of `error_word`. */
int chroma_b200_gemm_bf16(const void* a, const void* b, const void* bias, const void* residual, void* c, int32_t m,
                          int32_t n, int32_t k, int32_t epilogue, float swiglu_alpha, float swiglu_limit, int32_t groups,
                          const int32_t* offsets, void* tile_scratch, unsigned int* error_word, void* stream, char* err,
                          size_t err_len);
/* Arena bytes of a program's executor (the manifest's workspace_bytes). */
int64_t chroma_b200_workspace_bytes(const chroma_b200_program* program);

/* Device-resident KV-cached decoding for a prefill/decode pair (the pair chroma.Decoder drives,
 * chroma/_src/decoder.py:44-152), for `batch` independent sequences. The cache [batch, L, ctx, KV, hd] stays in
 * device memory; masks are built on the device from each sequence's ring-slot positions with the semantics of
 * decoder.py:115-127. */
int chroma_b200_decoder_create(chroma_b200_program* prefill, chroma_b200_program* decode, int32_t sliding_window,
                               int32_t batch, chroma_b200_decoder** out, char* err, size_t err_len);
/* One chunk for every sequence: `tokens` [batch, steps] (steps = 1 for decode, the prefill width otherwise;
 * entries past `count` are padding), `positions` [batch] absolute position of each sequence's first token.
 * Writes the logits of row count-1 to `logits` [batch, V] (storage type) when non-NULL, and the greedy argmax
 * (lowest index on ties) to `argmax` [batch] when non-NULL. New K/V rows are staged, not committed. */
int chroma_b200_decoder_step(chroma_b200_decoder* decoder, int32_t use_decode, const int64_t* tokens, int32_t count,
                             const int64_t* positions, void* logits, int64_t* argmax, char* err, size_t err_len);
/* Writes rows [0, count) staged by the last step of the given program into ring slots (position % ctx) and
 * records their positions; `positions` [batch] are that step's first positions. Idempotent until the same
 * program steps again, so a host may commit lazily (decoder.py:130-137 commits only after a call succeeds). */
int chroma_b200_decoder_commit(chroma_b200_decoder* decoder, int32_t use_decode, int32_t count,
                               const int64_t* positions, char* err, size_t err_len);
/* Greedy generation entirely on the device: `steps` decode steps, each decoding every sequence's current token,
 * committing its K/V row, advancing its position and feeding its argmax back as the next token. With `tokens` and
 * `positions` ([batch] each) the first step consumes those; with NULL it continues from the device state a
 * previous advance left. Rows staged by a host step must be committed first. Queued on `stream` (0: the
 * decoder's own); when `ids` is non-NULL the generated ids [steps, batch] are copied there and the stream is
 * synchronised. */
int chroma_b200_decoder_advance(chroma_b200_decoder* decoder, const int64_t* tokens, const int64_t* positions,
                                int32_t steps, void* stream, int64_t* ids, char* err, size_t err_len);
/* Kernels launched by one `advance` step (launch accounting). */
int32_t chroma_b200_decoder_step_launches(const chroma_b200_decoder* decoder);
/* Queues the decode program's layers alone (embedding through the final norm: the one-launch cluster kernel for
 * batch-1 fp32 programs) on `stream`, for per-kernel event timing. */
int chroma_b200_decoder_launch_layers(chroma_b200_decoder* decoder, void* stream, char* err, size_t err_len);
/* Queues the decode program's vocab-projection kernel alone on `stream` (for per-kernel event timing). */
int chroma_b200_decoder_launch_vocab(chroma_b200_decoder* decoder, void* stream, char* err, size_t err_len);
/* Empties every sequence's cache. */
int chroma_b200_decoder_reset(chroma_b200_decoder* decoder, char* err, size_t err_len);
/* Copies the committed cache and slot positions to host buffers ([batch, L, ctx, KV, hd] twice, [batch, ctx]). */
int chroma_b200_decoder_read(chroma_b200_decoder* decoder, void* keys, void* values, int64_t* slots, char* err,
                             size_t err_len);
/* Inverse of decoder_read for sequences [first, first + count): writes their committed cache ([count, L, ctx, KV,
 * hd] keys and values in the cache's storage type) and slot positions ([count, ctx], -1 = empty). Host or device
 * pointers (unified addressing). Rows staged by a step and not yet committed must be committed first. For caches
 * restored from elsewhere and for synthetic benchmark caches. No reference counterpart (the reference passes the
 * whole cache in with every call, decoder.py:115-130). */
int chroma_b200_decoder_write(chroma_b200_decoder* decoder, int32_t first, int32_t count, const void* keys,
                              const void* values, const int64_t* slots, char* err, size_t err_len);
void chroma_b200_decoder_destroy(chroma_b200_decoder* decoder);

/* Page-locked host memory for results the caller keeps (the decoders' returned logits): device-to-host copies
 * into it run at full link speed without a driver staging copy. The reference returns fresh numpy arrays
 * (chroma/_src/decoder.py:130-138); the Python layer returns numpy arrays over these blocks. */
int chroma_b200_host_alloc(size_t bytes, void** out, char* err, size_t err_len);
void chroma_b200_host_free(void* p);

/* ---- Expert parallelism across the GPUs of one node ---------------------------------------------------------------
 * No reference counterpart: the reference runs every expert on one device (the MoE einsums of
 * chroma/models/gpt_oss.py:243-265 lowered by chroma/_src/codegen/gpu.py:390-424). Here rank r of a group of `world`
 * processes (one GPU each) owns experts [r*E/world, (r+1)*E/world) and exchanges the routed rows with the other ranks
 * through their device memory (NVLink peer stores, no host round trip, capturable in CUDA graphs).
 *
 * Setup, once per process: create the group on the current device, export this rank's handle, gather every rank's
 * handle in rank order through any host channel (e.g. torch.distributed), open them. Then create programs with
 * chroma_b200_create_ep: their weights hold the local experts only (tensors 9-12 of each layer with E/world experts;
 * the router weights stay [E, d]). All ranks must run the same programs in the same order: every MoE layer waits
 * (bounded, ~1 s) for all ranks; a rank that does not arrive turns into a RUNTIME error on the others. */
#define CHROMA_B200_EP_HANDLE_BYTES 64
typedef struct chroma_b200_ep chroma_b200_ep;
/* `max_pairs`: the most (token, expert) pairs one call of any program on this rank routes (rows x top_k).
 * `vocab_rows` > 0 also splits the vocab projection by vocab rows (column shard of the logits): rank r holds
 * unembedding rows [r*ceil(V/world), ...) (tensor [2] of its programs has only those rows), every rank projects all
 * ranks' final rows onto its shard, and each row's owner receives the shards' argmax keys (and logits when a call
 * returns logits). `vocab_rows` is the most final rows one call selects on a rank; `vocab` = V (a multiple of 8).
 * 0 keeps the vocab projection replicated. */
int chroma_b200_ep_create(int32_t rank, int32_t world, int64_t max_pairs, int32_t hidden, int32_t experts,
                          int32_t vocab_rows, int32_t vocab, chroma_b200_ep** out, char* err, size_t err_len);
/* Writes CHROMA_B200_EP_HANDLE_BYTES bytes identifying this rank's shared buffer to other processes. */
int chroma_b200_ep_handle(const chroma_b200_ep* ep, void* handle, char* err, size_t err_len);
/* `handles`: world x CHROMA_B200_EP_HANDLE_BYTES bytes, every rank's handle in rank order. */
int chroma_b200_ep_open(chroma_b200_ep* ep, const void* handles, char* err, size_t err_len);
/* The group stays alive while programs created on it do. */
void chroma_b200_ep_destroy(chroma_b200_ep* ep);
/* chroma_b200_create (weights_path) or chroma_b200_create_device (device_weights) for an expert-parallel program:
 * exactly one of the two is non-NULL. */
int chroma_b200_create_ep(const chroma_b200_desc* desc, const char* weights_path, const void* device_weights,
                          chroma_b200_ep* ep, chroma_b200_program** out, char* err, size_t err_len);

#ifdef __cplusplus
}
#endif
#endif
