/*
 * oracle.h -- CPU restatement of ChatNet's quantized-weight hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for
 * libchatnet_cuda and the timed CPU baseline ("port") in bench.py.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs load it.  The
 * product library never links or calls it.
 *
 * Every function restates one C# routine of the reference (paths relative
 * to the ChatNet source tree) with the same per-operation rounding order:
 *   - fp16 decode            Tensors/Quantization/DequantQ4_0.cs:190-194
 *   - Q4_0 Dequantize / Dot  DequantQ4_0.cs:28-58, :80-149
 *   - Q4_K Dequantize / Dot  DequantQ4K.cs:37-77, :89-163, scales :218-264
 *   - Q6_K Dequantize / Dot  DequantQ6K.cs:37-88, :104-188
 *   - MatVecMul*             Tensors/TensorMath.cs:548-656 (row split >= 512)
 *   - RmsNorm / Softmax / SiluElementwiseMul / ApplyRoPE / Add
 *                            TensorMath.cs:97-165, :177-241, :253-286,
 *                            :408-458, :712-733
 *   - attention / forward    Models/Llama/LlamaModel.cs:241-346, :93-238,
 *                            embedding :365-394
 *   - greedy argmax          Samplers/GreedySampler.cs:13-26
 *   - tensor byte sizes      Gguf/GgufTensorInfo.cs:30-114
 *
 * Parity pin: the Q4_0 / Q4_K / Q6_K known-answer tests of
 * tests/ChatNet.Tests/QuantizationTests.cs (tests/golden/kat_quant.json).
 * The reference is C# (net10.0) and no .NET toolchain exists on either
 * machine, so nothing else is pinned by running the reference; RoPE,
 * attention and the forward pass rest on this line-by-line restatement.
 *
 * Vector widths: Vector128<float> is 4 lanes; Vector<float> is taken as
 * 8 lanes (x86-64 with AVX2, the width .NET picks there by default).
 * Lane order and the horizontal sums follow the reference: Vector128.Sum is
 * (v0+v1)+(v2+v3); TensorMath.VectorSum and LlamaModel.VectorSumFast add
 * lanes 0..7 in order.  Compiled with -ffp-contract=off (RyuJIT does not
 * contract a*b+c into an FMA).
 */
#ifndef CHATNET_ORACLE_H
#define CHATNET_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GgmlType values (Gguf/GgufConstants.cs:41-71). */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7, OR_Q8_0 = 8,
       OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14, OR_Q8_K = 15,
       OR_IQ2_XXS = 16, OR_IQ2_XS = 17, OR_IQ3_XXS = 18, OR_IQ1_S = 19, OR_IQ4_NL = 20, OR_IQ3_S = 21,
       OR_IQ2_S = 22, OR_IQ4_XS = 23, OR_IQ1_M = 29 };

float or_half_to_float(uint16_t h);
uint16_t or_float_to_half(float f); /* IEEE round-to-nearest-even */

/* GgufTensorInfo.ByteSize for the supported types; 0 for unknown. */
uint64_t or_byte_size(int type, uint64_t elements);

/* Dequantize(ReadOnlySpan<byte>, Span<float>, int). */
int or_dequantize(int type, const uint8_t* src, float* dst, int64_t n);

/* DotProduct(byte*, float*, int) -- the Vector128 path. */
float or_dot(int type, const uint8_t* row, const float* x, int n);

/* MatVecMulByType (LlamaModel.cs:470-567): y[r] = Dot(W + r*bpr, x, inDim).
 * nthreads <= 0 uses all cores; rows are split only when outDim >= 512,
 * like Parallel.For in TensorMath.  Returns 0, or -2 for an unsupported
 * type (the reference throws NotSupportedException). */
int or_matvec(int type, const uint8_t* W, const float* x, float* y,
              int out_dim, int in_dim, int nthreads);
/* batch of independent matvecs: x [batch][in_dim], y [batch][out_dim] */
int or_matvec_batch(int type, const uint8_t* W, const float* x, float* y,
                    int out_dim, int in_dim, int batch, int nthreads);

void or_rmsnorm(const float* x, const float* w, float* y, int n, float eps);
void or_softmax(float* data, int length);
void or_silu_mul(float* gate, const float* up, int length);
void or_rope(float* q, float* k, int pos, int head_dim, int n_heads,
             int n_kv_heads, float freq_base);
void or_add(float* a, const float* b, int length);
/* Architecture variants on the same loop: ApplyRoPENeox (split-half pairs),
 * GeluElementwiseMul, RmsNormWithOffset (TensorMath.cs:475, :294, :335). */
void or_rope_neox(float* q, float* k, int pos, int head_dim, int n_heads,
                  int n_kv_heads, float freq_base);
void or_gelu_mul(float* gate, const float* up, int length);
void or_rmsnorm_offset(const float* x, const float* w, float* y, int n, float eps);
int or_argmax(const float* logits, int n);
/* TemperatureSampler.Sample with the draw r given; *margin = distance of the
 * closest running sum to its threshold (top_p or r). */
int or_sample_temperature(const float* logits, int vocab, float temperature, int top_k, float top_p, float r,
                          float* margin);

/* Llama model restatement.  Tensors are passed as one flat array in the
 * order used by libchatnet_cuda's cn_llama_create:
 *   [0] token_embd  [1] output (may alias token_embd)  [2] output_norm
 *   then per layer l, base 3 + 9*l:
 *   attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm,
 *   ffn_gate, ffn_up, ffn_down
 * with types[] parallel to it (norm weights are OR_F32). */
typedef struct {
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, head_dim, vocab,
        ctx_len;
    float rope_base, eps;
    int kv_f16; /* 0: fp32 cache like the reference; 1: fp16 cache */
    int rope_neox, act_gelu, norm_offset; /* architecture variants, 0 = Llama */
} or_llama_config;

/* kcache / vcache: [n_layers][ctx_len][n_kv_heads*head_dim] of float or
 * uint16 (fp16) as cfg->kv_f16 says.  Runs Forward(tokens, pos, logits)
 * for one sequence: n tokens at positions pos..pos+n-1, logits for the
 * last one.  Returns 0 or a negative error. */
int or_llama_forward(const or_llama_config* cfg, const void* const* tensors,
                     const int* types, void* kcache, void* vcache,
                     const int* tokens, int n, int pos, float* logits,
                     int nthreads);

/* Forward for a subset of layers [l0, l1) starting from a given hidden
 * state x [dim] (used for layer-sampled CPU timing and prefill checks).
 * x is updated in place. */
int or_llama_layers(const or_llama_config* cfg, const void* const* tensors,
                    const int* types, void* kcache, void* vcache,
                    float* x, int pos, int l0, int l1, int nthreads);

/* Final norm + lm_head on hidden state x. */
int or_llama_head(const or_llama_config* cfg, const void* const* tensors,
                  const int* types, const float* x, float* logits,
                  int nthreads);

/* Seeded synthetic inputs of the benchmark configs (synth.cpp): the same
 * bytes as the product's generator (cn_synth_seed / cn_synth_fill), so CPU
 * legs never load the product library.  norm_weight selects 1 + 0.01*N for
 * F32.  Returns 0, -1 for a bad shape or size, -2 for a type without a
 * generator (only Q4_0, Q4_K, Q6_K, F32 and F16 have one). */
uint64_t or_synth_seed(int config_id, const char* name);
int or_synth_fill(int type, int64_t rows, int64_t cols, uint64_t seed,
                  int norm_weight, void* out, uint64_t bytes);
/* Rows [row0, row0 + rows) of what or_synth_fill would write for a tensor of
 * at least row0 + rows rows (the generator is counter-based). */
int or_synth_fill_rows(int type, int64_t row0, int64_t rows, int64_t cols,
                       uint64_t seed, int norm_weight, void* out,
                       uint64_t bytes);

#ifdef __cplusplus
}
#endif
#endif
