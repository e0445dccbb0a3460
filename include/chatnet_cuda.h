/*
 * chatnet_cuda.h -- C ABI of libchatnet_cuda, the B200 (sm_100a) engine for
 * ChatNet's quantized-weight hot path.
 *
 * The reference is a C# engine; its host code (InferenceEngine, IModel,
 * IWeightLoader) stays unchanged and reaches this library through
 * P/Invoke.  Every entry point below names the reference routine it
 * replaces (paths relative to the ChatNet source tree).
 *
 * Conventions
 *  - Every function returns int status: CN_OK (0) or a negative CN_ERR_*.
 *    Nothing throws or aborts.  cn_last_error() returns a message for the
 *    last failing call on the calling thread.
 *  - Status codes stand for the reference's exceptions:
 *    CN_ERR_UNSUPPORTED = NotSupportedException (LlamaModel.cs:564-565),
 *    CN_ERR_NOT_FOUND   = KeyNotFoundException (MemoryMappedWeights.cs:52),
 *    CN_ERR_INVALID_ARG = ArgumentException / IndexOutOfRangeException.
 *  - "_dev" entry points take DEVICE pointers and a cudaStream_t passed as
 *    void* (NULL = legacy default stream); they only enqueue work.
 *  - Entry points without "_dev" take HOST pointers, borrowed for the call,
 *    and return when the results are in host memory (the drop-in shape of
 *    the reference's synchronous Span-based methods).
 *  - Weight tensors hold the GGUF block bytes exactly as they are in the
 *    file (uploaded once, untouched), row-major [rows][row_bytes].
 */
#ifndef CHATNET_CUDA_H
#define CHATNET_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CN_ABI_VERSION 2

/* status codes */
#define CN_OK 0
#define CN_ERR_INVALID_ARG (-1)
#define CN_ERR_UNSUPPORTED (-2)
#define CN_ERR_CUDA (-3)
#define CN_ERR_OOM (-4)
#define CN_ERR_TIMEOUT (-5)
#define CN_ERR_NOT_FOUND (-6)
#define CN_ERR_NCCL (-7)

/* GgmlType values (Gguf/GgufConstants.cs:41-71) of the supported types. */
#define CN_TYPE_F32 0
#define CN_TYPE_F16 1
#define CN_TYPE_Q4_0 2
#define CN_TYPE_Q4_1 3
#define CN_TYPE_Q5_0 6
#define CN_TYPE_Q5_1 7
#define CN_TYPE_Q8_0 8
#define CN_TYPE_Q2_K 10
#define CN_TYPE_Q3_K 11
#define CN_TYPE_Q4_K 12
#define CN_TYPE_Q5_K 13
#define CN_TYPE_Q6_K 14
#define CN_TYPE_Q8_K 15
#define CN_TYPE_IQ2_XXS 16
#define CN_TYPE_IQ2_XS 17
#define CN_TYPE_IQ3_XXS 18
#define CN_TYPE_IQ1_S 19
#define CN_TYPE_IQ4_NL 20
#define CN_TYPE_IQ3_S 21
#define CN_TYPE_IQ2_S 22
#define CN_TYPE_IQ4_XS 23
#define CN_TYPE_IQ1_M 29

typedef struct cn_ctx cn_ctx;
typedef struct cn_tensor cn_tensor;

/* ---- library ------------------------------------------------------------ */

/* Returns CN_ABI_VERSION.  (no reference counterpart: ABI handshake) */
int cn_abi_version(void);

/* Message for the last failing call on this thread ("" if none).  The
 * pointer stays valid until the next failing call on the same thread.
 * (stands for Exception.Message) */
const char* cn_last_error(void);

/* Bytes of `elements` values stored as `type`; 0 for unsupported types.
 * Replaces GgufTensorInfo.ByteSize (Gguf/GgufTensorInfo.cs:30-114). */
uint64_t cn_byte_size(int type, uint64_t elements);

/* Number of visible CUDA devices. */
int cn_device_count(int* out_count);

/* ---- context ------------------------------------------------------------ */

/* Creates a context on `device` with one stream and the scratch space the
 * kernels need.  Replaces the per-model state LlamaModel allocates in its
 * constructor (LlamaModel.cs:48-73). */
int cn_create(int device, cn_ctx** out);
int cn_destroy(cn_ctx* ctx);
/* The context's cudaStream_t (as void*). */
void* cn_ctx_stream(cn_ctx* ctx);
/* Waits for the context's stream; also reports a device-side timeout
 * (CN_ERR_TIMEOUT) if a kernel gave up waiting. */
int cn_synchronize(cn_ctx* ctx);

/* ---- weight tensors -------------------------------------------------- */

/* Uploads `bytes` of GGUF blocks for a [rows, cols] tensor of `type` to
 * HBM, byte for byte.  bytes must equal rows * cn_byte_size(type, cols).
 * Replaces MemoryMappedWeights.GetTensorPointer/GetTensorData
 * (Memory/MemoryMappedWeights.cs:48-83) as the source of weight bytes. */
int cn_tensor_upload(cn_ctx* ctx, const void* host_blocks, uint64_t bytes, int type,
                     int64_t rows, int64_t cols, cn_tensor** out);

/* Uploads the region [row0, row0 + nrows) x [col0, col0 + ncols) of a host
 * tensor of rows x cols (bytes = rows * cn_byte_size(type, cols), e.g. the
 * pointer MemoryMappedWeights.GetTensorPointer returns, Memory/
 * MemoryMappedWeights.cs:76) as a tensor of its own: a tensor-parallel rank's
 * shard.  Columns must cover whole blocks (32 or 256 weights); the rows are
 * copied with one strided copy, no host staging.  (no reference
 * counterpart: the reference runs on one CPU) */
int cn_tensor_upload_slice(cn_ctx* ctx, const void* host_blocks, uint64_t bytes, int type, int64_t rows,
                           int64_t cols, int64_t row0, int64_t nrows, int64_t col0, int64_t ncols,
                           cn_tensor** out);

/* Allocates a tensor and fills it on the device with the seeded synthetic
 * generator (cn_synth_fill); no host copy.  (no reference counterpart:
 * synthetic inputs for the benchmark configs) */
int cn_tensor_synth(cn_ctx* ctx, int type, int64_t rows, int64_t cols, uint64_t seed,
                    int dist, cn_tensor** out);

/* Like cn_tensor_synth, but allocates and fills only the region
 * [row0, row0 + nrows) x [col0, col0 + ncols) of the rows x cols tensor that
 * cn_tensor_synth would produce (columns in whole blocks): a tensor-parallel
 * rank generates its own shard.  (no reference counterpart: synthetic
 * inputs) */
int cn_tensor_synth_slice(cn_ctx* ctx, int type, int64_t rows, int64_t cols, int64_t row0,
                          int64_t nrows, int64_t col0, int64_t ncols, uint64_t seed, int dist,
                          cn_tensor** out);

/* Copies a tensor's bytes back to host memory (bytes must match). */
int cn_tensor_download(const cn_tensor* t, void* host, uint64_t bytes);
int cn_tensor_free(cn_tensor* t);
const void* cn_tensor_device_ptr(const cn_tensor* t);
uint64_t cn_tensor_bytes(const cn_tensor* t);

/* ---- synthetic inputs (host side; identical bytes on the device) -------- */

/* Distributions for cn_synth_fill / cn_tensor_synth. */
#define CN_DIST_CFG0_Q4_0 1  /* Q4_0, d = |N|*0.02/8, nibbles U[0,15]          */
#define CN_DIST_CFG2_Q4_K 2  /* Q4_K, d,dmin = |N|*0.01, 6-bit sc/m U[0,63]    */
#define CN_DIST_CFG2_Q6_K 3  /* Q6_K, d = |N|*0.01, int8 scales U[0,63]        */
#define CN_DIST_NORMAL 4     /* F32 or F16: N(0,1)                              */
#define CN_DIST_NORM_W 5     /* F32: 1 + 0.01*N(0,1) (RMSNorm weights)          */

/* Fills `host` with the generator's bytes for a [rows, cols] tensor.
 * N(0,1) is the sum of twelve 16-bit uniforms minus 6, exact in fp32.
 * (no reference counterpart) */
int cn_synth_fill(int type, int64_t rows, int64_t cols, uint64_t seed, int dist, void* host,
                  uint64_t bytes);
/* 64-bit seed of a named tensor in a benchmark config (FNV-1a of the name
 * mixed with the config id). */
uint64_t cn_synth_seed(int config_id, const char* tensor_name);

/* ---- op level: host buffers, synchronous -------------------------------- */

/* Dequantizes rows [row0, row0+nrows) of W to fp32, bit-exact with
 * DequantQ4_0/Q4K/Q6K.Dequantize (Tensors/Quantization/DequantQ4_0.cs:28-58,
 * DequantQ4K.cs:37-77, DequantQ6K.cs:37-88). */
int cn_dequantize(cn_ctx* ctx, const cn_tensor* W, int64_t row0, int64_t nrows, float* host_out);

/* y[b][r] = dot(W[r], x[b]) for b < batch: x is [batch][cols] fp32, y is
 * [batch][rows] fp32.  Replaces MatVecMulByType (Models/Llama/
 * LlamaModel.cs:470-567) -> TensorMath.MatVecMulQ4_0 / MatVecMulQ6K /
 * MatVecMulGeneric(Q4_K) (Tensors/TensorMath.cs:548-656). */
int cn_matvec(cn_ctx* ctx, const cn_tensor* W, const float* host_x, float* host_y, int batch);

/* Prefill matmul: y[t][r] = dot(W[r], x[t]) for n_tokens tokens at once (x
 * [n_tokens][cols] fp32, y [n_tokens][rows] fp32), the batched form of the
 * matvec that ChatNet runs once per prompt token (InferenceEngine.cs:235-239
 * -> TensorMath.MatVecMulQ4_0 / MatVecMulGeneric(Q4_K), Tensors/TensorMath.cs:
 * 548-578, 624-656).  Runs on the tcgen05 tensor cores: each token's row
 * scaled by a power of two and rounded to fp16, weights expanded to fp16,
 * fp32 accumulation.  Q4_0 or Q4_K weights with cols % 256 == 0; other
 * types return CN_ERR_UNSUPPORTED. */
int cn_matmul(cn_ctx* ctx, const cn_tensor* W, const float* host_x, float* host_y, int n_tokens);

/* ---- device level: device pointers, asynchronous ------------------------ */

/* Bit-exact dequantization of n_elements values (same semantics as the
 * reference Dequantize, including Q4_0's partial last block and the K
 * types' whole-super-block rule). */
int cn_dequantize_dev(int type, const void* d_blocks, float* d_out, int64_t n_elements,
                      void* stream);

/* Fused dequant-GEMV on raw device pointers, using ctx's scratch and
 * stream: y[b][r] = dot(W[r], x[b]).  Same math as cn_matvec. */
int cn_matvec_dev(cn_ctx* ctx, int type, const void* d_w, int out_dim, int in_dim,
                  const float* d_x, float* d_y, int batch);

/* Measurement hook for the op-level GEMV (bench.py's GB/s lines): captures
 * `launches` calls of cn_matvec_dev's work (x-prep + fused GEMV) cycling
 * through the n_w same-shaped matrices ws (distinct copies keep L2 cold),
 * replays the graph `reps` times on ctx's stream and writes each replay's
 * mean microseconds per call to us_out[reps].  *kernels_per_launch = kernels
 * one call launches.  (no counterpart in the reference: timing only) */
int cn_time_matvec(cn_ctx* ctx, const cn_tensor* const* ws, int n_w, const float* d_x, float* d_y,
                   int batch, int launches, int reps, float* us_out, int* kernels_per_launch);

/* cn_llama_sample on caller-owned device logits [batch][vocab] (ctx's stream;
 * returns when tokens_host is written). */
int cn_sample_dev(cn_ctx* ctx, const float* d_logits, int vocab, int batch, float temperature, int top_k,
                  float top_p, const float* r_host, int* tokens_host);

/* Prefill matmul of cn_matmul on device pointers, using ctx's scratch and
 * stream (enqueued; no synchronisation). */
int cn_matmul_dev(cn_ctx* ctx, int type, const void* d_w, int out_dim, int in_dim,
                  const float* d_x, float* d_y, int n_tokens);

/* The fused dequant-GEMV of cn_matvec_dev for callers that cannot allocate
 * device memory (hosts that own every buffer, or forbid cudaMalloc/cudaFree
 * once running): no context, no allocation.  Its scratch is one fixed 4 MiB
 * array inside the library, present on every GPU that loads it; calls needing
 * more are rejected with CN_ERR_INVALID_ARG (batch 1..4 fits inner dimensions
 * beyond 100k).  Calls share that array, so calls whose GPU work overlaps
 * race: serialise them.  The first call on each device (and the first after
 * a cudaDeviceReset) looks up the array's address and must not happen during
 * a stream capture.  `stream` is a cudaStream_t (NULL = legacy default
 * stream); the call only enqueues work.
 * (no counterpart in the reference: an allocation-free variant of
 * cn_matvec_dev) */
int cn_matvec_noalloc_dev(int type, const void* d_w, int out_dim, int in_dim, const float* d_x,
                          float* d_y, int batch, void* stream);
/* Waits for `stream`, then reads and clears the no-alloc array's device error
 * word: CN_ERR_TIMEOUT if a cn_matvec_noalloc_dev kernel since the last
 * check gave up waiting (its y is then incomplete), CN_OK otherwise.
 * Allocates nothing.  (no counterpart in the reference: the error report of
 * the allocation-free GEMV) */
int cn_matvec_noalloc_status(void* stream);

/* ---- model level: one Llama decoder resident on the device ------------- */

typedef struct cn_llama cn_llama;

#define CN_KV_F32 0 /* fp32 KV cache, as LlamaModel allocates (LlamaModel.cs:60-61) */
#define CN_KV_F16 1 /* fp16 KV cache (rounded to nearest on store)                  */

/* Hyper-parameters; mirrors LlamaConfig (Models/Llama/LlamaConfig.cs:23-39). */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab, ctx_len;
    float rope_base, rms_eps;
    int kv_dtype;  /* CN_KV_F32 or CN_KV_F16 */
    int max_batch; /* sequences decoded together, 1..32; each owns a KV slot */
    /* Variants other ChatNet models run on the same loop (0 = Llama):
     * rope_neox   split-half RoPE pairs (i, i + head_dim/2), TensorMath.ApplyRoPENeox
     *             (Tensors/TensorMath.cs:475; Qwen/Phi), instead of interleaved pairs;
     * act_gelu    GELU(gate) * up, TensorMath.GeluElementwiseMul (TensorMath.cs:294;
     *             Gemma), instead of SiLU(gate) * up;
     * norm_offset RMSNorm weights stored as (weight - 1), TensorMath.RmsNormWithOffset
     *             (TensorMath.cs:335; Gemma). */
    int rope_neox, act_gelu, norm_offset;
} cn_llama_config;

/* Number of tensors cn_llama_create takes for n_layers layers. */
#define CN_LLAMA_TENSORS(n_layers) (3 + 9 * (n_layers))

/* Builds the model from uploaded tensors (borrowed: they must outlive the
 * model), in the order LlamaWeights.ResolveAll resolves them
 * (Models/Llama/LlamaWeights.cs:78-145):
 *   [0] token_embd [rows=vocab, cols=dim]
 *   [1] output     [vocab, dim]  (pass token_embd again when the file has no
 *                                 output.weight, LlamaWeights.cs:89-98)
 *   [2] output_norm F32 [1, dim]
 *   then for each layer l, at 3 + 9*l:
 *   attn_norm F32 [1, dim], attn_q [dim, dim], attn_k [kv, dim],
 *   attn_v [kv, dim], attn_output [dim, dim], ffn_norm F32 [1, dim],
 *   ffn_gate [hidden, dim], ffn_up [hidden, dim], ffn_down [dim, hidden]
 * Allocates the KV cache ([max_batch][layers][ctx][kv] zero-filled, like
 * LlamaModel.cs:60-61) and all scratch.  Replaces the LlamaModel
 * constructor (LlamaModel.cs:48-88). */
int cn_llama_create(cn_ctx* ctx, const cn_llama_config* cfg, cn_tensor* const* tensors,
                    int n_tensors, cn_llama** out);
int cn_llama_destroy(cn_llama* m);

/* IModel.Forward (Abstractions/IModel.cs:18, LlamaModel.cs:93-238): runs the
 * n tokens of KV slot 0 at positions pos..pos+n-1 and writes the logits of
 * the last one to logits_host [vocab].  A prompt of 16 or more tokens (the
 * threshold cn_llama_set_prefill sets) runs as one prefill pass when the
 * model supports it (cn_llama_prefill_hidden_dev); shorter ones, and models
 * the pass cannot run, take one decode step per token as the reference does
 * (InferenceEngine.cs:235-239). */
int cn_llama_forward(cn_llama* m, const int* tokens, int n, int pos, float* logits_host);

/* Prompts of min_tokens (>= 16; 16 by default) or more tokens in
 * cn_llama_forward run as one prefill pass on a one-GPU model whose
 * projections are Q4_0, Q4_K or Q6_K (every layer on the tcgen05 matmul for
 * all n tokens, see cn_llama_prefill_hidden_dev; a Q6_K matrix whose rows are
 * not 16-byte multiples, such as Llama-2-7B's ffn_down at 11008 columns, runs
 * from a row-padded copy the model makes at creation); 0 turns
 * it off, so every prompt token runs as a decode step.  (no reference
 * counterpart: the reference has only the sequential loop) */
int cn_llama_set_prefill(cn_llama* m, int min_tokens);

/* Precision of the prefill pass (hidden states against the reference's
 * sequential fp32 steps, one layer, trained-model-like Q4_K_M weights:
 * measured worst token / median).
 *   2 (the default): every projection carries weights and activations as
 *     exact pairs of fp16 halves (three MMAs per k-step) and the attention
 *     uses q, k (and, for fp32 caches, v) and its output the same way:
 *     near-fp32 results, 2-3e-4 / 1-2e-4, about 2x the matmul time of 0;
 *   1: only the attention path (q/k/v and O projections, attention) split,
 *     the feed-forward matmuls on fp16 operands: ~1e-3 / 7e-4;
 *   0: every operand rounded to fp16 once (fastest): ~2e-3 / 1.4e-3, and on
 *     ill-conditioned inputs (a peaked softmax, tokens at the SwiGLU knee)
 *     up to a few 1e-2.
 * (no reference counterpart) */
int cn_llama_set_prefill_precision(cn_llama* m, int split);

/* Prefill on device buffers: runs the hidden states x_dev [n][dim] (fp32)
 * through every layer at once, for positions pos..pos+n-1 of KV slot 0 (whose
 * cache rows are written), and writes the layer stack's output to out_dev
 * [n][dim] (may equal x_dev).  Enqueued on the context stream, not waited
 * for.  Needs Q4_0 projections, dim and hidden_dim multiples of 256, head_dim
 * 64 or 128, and one GPU (CN_ERR_UNSUPPORTED otherwise).
 * (no counterpart in the reference: the per-layer part of LlamaModel.Forward,
 * Models/Llama/LlamaModel.cs:93-238, for n tokens at once) */
int cn_llama_prefill_hidden_dev(cn_llama* m, const float* x_dev, int n, int pos, float* out_dev);
/* Kernel launches of one cn_llama_prefill_hidden_dev call. */
int cn_llama_prefill_kernels(cn_llama* m, int* n_kernels);

/* One decode step for `batch` sequences: sequence b (KV slot b) reads token
 * tokens[b] at position pos[b].  logits_host [batch][vocab] and argmax_host
 * [batch] (GreedySampler.Sample, Samplers/GreedySampler.cs:13-26) may each
 * be NULL.  The step runs as a CUDA graph captured on the first call for
 * each batch size, so that first call must not happen during a stream
 * capture. */
int cn_llama_decode(cn_llama* m, const int* tokens, const int* pos, int batch, float* logits_host,
                    int* argmax_host);

/* Sets the step inputs (token ids and positions of `batch` sequences) in
 * device memory, then cn_llama_step enqueues one decode step on the
 * context's stream without any host copy or wait; the logits and argmax stay
 * on the device.  Together they split cn_llama_decode for callers that keep
 * the loop on the device (benchmarks, device-side sampling).  The first
 * cn_llama_step of each batch size captures the CUDA graph. */
int cn_llama_set_inputs(cn_llama* m, const int* tokens, const int* pos, int batch);
int cn_llama_step(cn_llama* m, int batch);

/* TemperatureSampler.Sample (Samplers/TemperatureSampler.cs:33-113) on the
 * device, for the logits the last decode step left there (sequences
 * 0..batch-1): logits * (1 / temperature), softmax, the top_k largest
 * probabilities in descending order cut at the first running sum >= top_p,
 * renormalised, then the first entry whose running sum exceeds r_host[b] --
 * the caller's Random.NextDouble() draw, so the host keeps the reference's
 * random stream.  temperature <= 0 returns the argmax (first maximum).
 * top_k must be >= 1 when sampling.  tokens_host [batch].  Probabilities
 * match the reference's to fp32 rounding (the softmax sum runs as a tree),
 * so a draw within rounding of a boundary may pick the neighbouring entry. */
int cn_llama_sample(cn_llama* m, int batch, float temperature, int top_k, float top_p, const float* r_host,
                    int* tokens_host);
/* Kernel launches one decode step makes for `batch` (nodes of its graph). */
int cn_llama_step_kernels(cn_llama* m, int batch, int* out_count);
/* Times one projection's fused dequant-GEMV as the step runs it (activation
 * prep excluded): `iters` launches cycling through the layers' matrices of
 * projection `proj` (0..6 = q,k,v,o,gate,up,down; 7 = lm_head; 8 = the q/k/v
 * and 9 = the gate/up matrices as the one grouped launch the step runs, or
 * CN_ERR_UNSUPPORTED where the model runs them apart), with CUDA events on
 * the context's stream.  Reports the mean time per launch and the launch's
 * algorithmic bytes (weights + x + y).  (no reference counterpart: roofline
 * measurement) */
int cn_llama_time_gemv(cn_llama* m, int proj, int batch, int iters, float* us_per_launch,
                       double* bytes_per_launch);
/* Runs one decode step for `batch` without its graph, recording an event
 * after each stage, and adds each stage's time (us) into us_by_stage[kind]
 * (kinds: 0 unused, 1 tensor-parallel step counter, 2 embedding, 3 add +
 * RmsNorm + prep, 4 q/k/v, 5 RoPE + KV store, 6 attention, 7 O, 8 gate/up,
 * 9 SiLU + prep, 10 down, 11 lm_head, 12 exchange wait, 13 argmax; at most
 * n_stages entries are written).  Events between launches serialise them, so
 * the sum exceeds the graph's step time.  (no reference counterpart:
 * diagnostics) */
int cn_llama_profile_step(cn_llama* m, int batch, float* us_by_stage, int n_stages);
/* Times one prefill matmul launch for n tokens as cn_llama_prefill_hidden_dev
 * runs it: group 0 = q/k/v (one launch), 1 = O, 2 = gate/up (one launch),
 * 3 = down; `iters` launches cycling through the layers, CUDA events on the
 * context's stream.  Reports the mean time per launch and its FLOPs
 * (2 * n * rows * cols).  Overwrites the prefill scratch.  (no reference
 * counterpart: roofline measurement) */
int cn_llama_time_matmul(cn_llama* m, int group, int n, int iters, float* us_per_launch,
                         double* flops_per_launch);

/* ---- GGUF files ------------------------------------------------------------ */

typedef struct cn_gguf cn_gguf;

/* GgufReader.Load (Gguf/GgufReader.cs:34-75) with the mapping of
 * MemoryMappedWeights (Memory/MemoryMappedWeights.cs:23-40): parses a GGUF
 * version 2 or 3 file (metadata, tensor descriptors, data section aligned to
 * general.alignment, default 32) and maps it read-only.  Bad magic, version
 * or a truncated header: CN_ERR_INVALID_ARG (InvalidDataException); a file
 * that cannot be opened: CN_ERR_NOT_FOUND. */
int cn_gguf_open(const char* path, cn_gguf** out);
int cn_gguf_close(cn_gguf* g);
int cn_gguf_tensor_count(const cn_gguf* g, int* n);
/* Tensor i's descriptor (GgufTensorInfo): name (valid until cn_gguf_close),
 * ggml type, dimensions (dims[0] innermost; 4 entries, unused ones 1), byte
 * size (GgufTensorInfo.ByteSize) and absolute offset in the file.  Any output
 * pointer may be NULL. */
int cn_gguf_tensor_info(const cn_gguf* g, int i, const char** name, int* type, int* n_dims,
                        uint64_t* dims, uint64_t* bytes, uint64_t* file_offset);
/* Index of a tensor by name; CN_ERR_NOT_FOUND ("Tensor not found: ...") otherwise. */
int cn_gguf_find(const cn_gguf* g, const char* name, int* index);
/* Metadata values (GgufMetadata.GetInt32 / TryGet / GetString). */
int cn_gguf_get_int(const cn_gguf* g, const char* key, int64_t* out);
int cn_gguf_get_float(const cn_gguf* g, const char* key, double* out);
int cn_gguf_get_string(const cn_gguf* g, const char* key, const char** out);
/* GgufReader.ExtractModelConfig (GgufReader.cs:80-176) for a Llama decoder:
 * <arch>.embedding_length, block_count, attention.head_count(_kv),
 * feed_forward_length, context_length, rope.freq_base,
 * attention.layer_norm_rms_epsilon, attention.key_length (head_dim, else
 * dim / heads), vocabulary = length of tokenizer.ggml.tokens, else
 * <arch>.vocab_size, with the reader's defaults and bare-key fallbacks.
 * kv_dtype = CN_KV_F32, max_batch = 1.  Architectures the reference runs with
 * another decoder (ModelFactory.cs:23-39): CN_ERR_UNSUPPORTED. */
int cn_gguf_llama_config(const cn_gguf* g, cn_llama_config* cfg);
/* Uploads one tensor byte for byte (cn_tensor_upload, [rows = product of
 * dims[1..], cols = dims[0]]). */
int cn_gguf_upload(cn_ctx* ctx, const cn_gguf* g, const char* name, cn_tensor** out);
/* LlamaWeights.ResolveAll (Models/Llama/LlamaWeights.cs:78-145) + the
 * LlamaModel constructor: uploads every tensor cn_llama_create needs (an
 * absent output.weight means lm_head tied to token_embd.weight) and builds
 * the model with the file's config, max_batch and kv_dtype.  The uploaded
 * tensors go to tensors_out (CN_LLAMA_TENSORS(n_layers) entries, the tied
 * lm_head repeating token_embd); free each distinct one with cn_tensor_free
 * after cn_llama_destroy. */
int cn_llama_create_from_gguf(cn_ctx* ctx, const cn_gguf* g, int max_batch, int kv_dtype,
                              cn_llama** out, cn_tensor** tensors_out, int n_tensors_out);
/* cn_llama_create_from_gguf for tensor-parallel rank tp->rank of tp->size
 * (a connected group, see below): uploads only this rank's shard of every
 * projection straight from the mapped file (cn_tensor_upload_slice; a tied
 * lm_head takes this rank's vocabulary rows of token_embd) and builds the
 * rank's model with cn_llama_create_tp.  (no reference counterpart) */
typedef struct cn_tp cn_tp;
int cn_llama_create_from_gguf_tp(cn_ctx* ctx, const cn_gguf* g, cn_tp* tp, int max_batch, int kv_dtype,
                                 cn_llama** out, cn_tensor** tensors_out, int n_tensors_out);

/* ---- tensor parallelism (one process per GPU) ---------------------------
 * (no reference counterpart: the reference runs on one CPU.)  Rank r of a
 * group of `size` GPUs holds shards of every projection: q/k/v/gate/up and
 * lm_head rows (r-th contiguous slice of heads, FFN rows, vocabulary), O and
 * down columns (r-th slice of their input).  The partial outputs of O and
 * down, and the lm_head slices, are exchanged inside the GEMV epilogue:
 * every value is stored straight into each rank's buffer over NVLink (CUDA
 * IPC), and the consumer kernel waits for every rank's flag.  Usage: every
 * rank calls cn_tp_create, shares cn_tp_handle's bytes with the others (any
 * host channel), calls cn_tp_connect with all ranks' handles in rank order,
 * then cn_llama_create_tp.  All ranks must then run the same sequence of
 * steps; a rank that stops makes the others' kernels give up after ~2 s
 * (CN_ERR_TIMEOUT), after which the group must be rebuilt. */
#define CN_TP_HANDLE_BYTES 64
int cn_tp_create(cn_ctx* ctx, int rank, int size, int max_batch, int dim, int vocab, cn_tp** out);
int cn_tp_handle(const cn_tp* tp, void* handle_out /* CN_TP_HANDLE_BYTES */);
int cn_tp_connect(cn_tp* tp, const void* handles /* size * CN_TP_HANDLE_BYTES, rank order */);
int cn_tp_destroy(cn_tp* tp);
/* cn_llama_create for rank tp->rank of a tensor-parallel group: cfg is the
 * whole model's; the tensors are this rank's shards (shapes as for
 * cn_llama_create with n_heads, n_kv_heads, hidden_dim and vocab divided by
 * the group size for the sharded dimensions).  The exchanged projections
 * must run on the integer Q4_K GEMV (Q4_K weights, max_batch <= 8). */
int cn_llama_create_tp(cn_ctx* ctx, const cn_llama_config* cfg, cn_tensor* const* tensors,
                       int n_tensors, cn_tp* tp, cn_llama** out);
/* Builds (and graph-captures) the step for `batch` sequences without running
 * it, so a tensor-parallel group can synchronise on the host before its
 * first step.  (no reference counterpart) */
int cn_llama_prepare(cn_llama* m, int batch);

/* KV cache access for seeding and checking (no reference counterpart; the
 * reference fills its cache only through Forward).  Element type follows
 * cfg.kv_dtype (float or uint16 fp16 bits), layout [npos][n_kv*head_dim]. */
int cn_llama_kv_write(cn_llama* m, int seq, int layer, int pos0, int npos, const void* k_host,
                      const void* v_host);
int cn_llama_kv_read(cn_llama* m, int seq, int layer, int pos0, int npos, void* k_host,
                     void* v_host);
/* Fills positions [0, npos) of every layer of KV slot `seq` with the seeded
 * N(0,1) generator (element index (layer*ctx + pos)*kv + d, as
 * cn_synth_fill lays out a [layers*ctx, kv] tensor) and zeroes the rest. */
int cn_llama_kv_synth(cn_llama* m, int seq, int npos, uint64_t seed_k, uint64_t seed_v);

#ifdef __cplusplus
}
#endif
#endif
