/*
 * muyo_cuda.h - the C-ABI of the B200 (sm_100a) decode-step kernel set.
 *
 * One shared library, libmuyo_cuda.so, replaces the reference's per-op Vulkan dispatches
 * (llama.cpp GLSL shaders driven by Muyo's RenderGraph) behind the reference's op-node interfaces.
 * Every entry point takes a POD parameter block carrying the same semantic fields as the
 * reference's push-constant block for that op (src/LlamaContracts.h), plain device pointers and a
 * CUDA stream (as `void*`, a cudaStream_t; NULL is the legacy default stream).
 *
 * Conventions (as in src/LlamaContracts.h:14-19): dimensions and strides are in ELEMENTS, not bytes,
 * most-minor dimension first. Buffers are owned by the caller; the op entry points allocate nothing.
 * Ops that need scratch take a caller-owned workspace and export a *_workspace_size query.
 *
 * Errors: every call returns MUYO_OK (0) or a negative MUYO_E* code and never throws; the message of
 * the last failure on the calling thread is muyo_cuda_last_error(). Arguments are validated before
 * any CUDA call, so a rejected call has no side effect. Kernel launches are asynchronous on the given
 * stream; device-side faults surface on a later synchronising call as MUYO_ECUDA.
 *
 * Reference citations are file:line within the muyo-llm project.
 */
#ifndef MUYO_CUDA_H
#define MUYO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ----------------------------------------------------------------------------------- */
#define MUYO_OK 0
#define MUYO_EINVAL (-1)       /* a shape, stride, pointer or alignment argument is invalid */
#define MUYO_ECUDA (-2)        /* a CUDA runtime call failed */
#define MUYO_ETIMEOUT (-3)     /* a bounded device-side wait gave up */
#define MUYO_ENOMEM (-4)       /* a set-up allocation failed (model create only) */
#define MUYO_EUNSUPPORTED (-5) /* a contract field the B200 kernels do not implement */
#define MUYO_ESTATE (-6)       /* call out of order (e.g. cache full, model not finalised) */

/* Replaces HeadlessContext's device bring-up (src/HeadlessContext.h:25-66): selects the CUDA
 * device for the calling thread and creates its primary context. */
int muyo_cuda_init(int device);
/* Replaces ~HeadlessContext: releases library-owned per-device state (never caller buffers). */
int muyo_cuda_shutdown(void);
/* Message of the last failing call on this thread ("" if none). */
const char* muyo_cuda_last_error(void);
/* Library version string ("muyo_cuda <semver> sm_100a"). */
const char* muyo_cuda_version(void);

/* ---- GEMV: mul_mat_vec ------------------------------------------------------------------------
 * Replaces MatVecExecute + mul_mat_vec_{f16,f32}_f32_f32 (src/FullModel.cpp:133-175,
 * shaders/llama/mul_mat_vec.comp, mul_mat_vec_base.glsl:49-100). Fields mirror
 * LlamaMatVecPushConstants (src/LlamaContracts.h:66-84) plus the dispatch the node issued:
 *   d[b*batch_stride_d + r] = sum_k A[ba*batch_stride_a + r*stride_a + k] * B[b*batch_stride_b + k]
 *                             (+ fuse0[b*batch_stride_d + r] if BIAS0) (+ fuse1[...] if BIAS1)
 * for r < rows, b < batches, with ba = (b / ne12 / broadcast3) * ne02 + (b % ne12) / broadcast2
 * (the GQA broadcast). FP32 accumulation. */
#define MUYO_MATVEC_BIAS0 0x1u
#define MUYO_MATVEC_BIAS1 0x2u
#define MUYO_MATVEC_SCALE0 0x4u /* accepted by the contract, not implemented: MUYO_EUNSUPPORTED */
#define MUYO_MATVEC_SCALE1 0x8u /* idem */

typedef struct MuyoMatVecParams {
    uint32_t ncols;    /* K */
    uint32_t stride_a; /* row stride of A (0 = ncols, as src/FullModel.cpp:158) */
    uint32_t stride_b; /* 0 = ncols */
    uint32_t stride_d; /* output row bound per batch (rows must not exceed it) */
    uint32_t batch_stride_a, batch_stride_b, batch_stride_d;
    uint32_t fusion_flags;
    uint32_t ne02, ne12, broadcast2, broadcast3; /* 0 is read as 1 */
    uint32_t rows;    /* rows computed (the node's dispatch x; src/FullModel.cpp:172) */
    uint32_t batches; /* the node's dispatch y (0 is read as 1) */
} MuyoMatVecParams;

/* A is F16 (IEEE binary16 bits). */
int muyo_cuda_mat_vec_f16(const MuyoMatVecParams* p, const void* a, const float* b, float* d, const float* fuse0,
                          const float* fuse1, void* stream);
/* A is F32 (the attention score / value GEMVs, src/FullModel.cpp:793-844). */
int muyo_cuda_mat_vec_f32(const MuyoMatVecParams* p, const float* a, const float* b, float* d, const float* fuse0,
                          const float* fuse1, void* stream);

/* ---- generic binary head (add, rms_norm, get_rows) ---------------------------------------------
 * Mirrors LlamaAddPushConstants (src/LlamaContracts.h:22-38) without the kernel-private
 * misalign_offsets: A = operand 0, B = operand 1, D = output; ne/nb most-minor first, elements. */
typedef struct MuyoBinaryParams {
    uint32_t ne; /* element count of D */
    uint32_t ne00, ne01, ne02, ne03, nb00, nb01, nb02, nb03;
    uint32_t ne10, ne11, ne12, ne13, nb10, nb11, nb12, nb13;
    uint32_t ne20, ne21, ne22, ne23, nb20, nb21, nb22, nb23;
    float param1; /* rms_norm: eps */
    float param2;
    int32_t param3;
} MuyoBinaryParams;

/* Replaces AddExecute + add.comp (src/FullModel.cpp:250-284): D = A + B, B repeated over A's
 * shape by modulo (ggml broadcast) when smaller. */
int muyo_cuda_add(const MuyoBinaryParams* p, const float* a, const float* b, float* d, void* stream);
/* Replaces RmsNormExecute + rms_norm.comp with do_multiply (src/FullModel.cpp:215-247):
 * each row of ne00 values: D = A * rsqrt(mean(A^2) + param1) * B[col % ne10]. */
int muyo_cuda_rms_norm(const MuyoBinaryParams* p, const float* a, const float* w, float* d, void* stream);
/* Replaces GetRowsExecute + get_rows_{f16_f32,f32} (src/FullModel.cpp:424-458):
 * D[i10, i11, i12][:] = float(A[B[i10, i11, i12], i11, i12][:]), B int32 row ids. */
int muyo_cuda_get_rows_f16(const MuyoBinaryParams* p, const void* a, const int32_t* b, float* d, void* stream);
int muyo_cuda_get_rows_f32(const MuyoBinaryParams* p, const float* a, const int32_t* b, float* d, void* stream);

/* ---- GLU (swiglu) -------------------------------------------------------------------------------
 * Mirrors LlamaGluPushConstants (src/LlamaContracts.h:182-199) minus the fastdiv magic. Replaces
 * SwigluExecute + swiglu.comp (src/FullModel.cpp:287-327): D = silu(gate) * up. mode 2 (split):
 * gate = A, up = B; mode 0: one A row holds [gate | up]; mode 1: [up | gate]. */
#define MUYO_GLU_HALVES 0u
#define MUYO_GLU_SWAPPED 1u
#define MUYO_GLU_SPLIT 2u
typedef struct MuyoGluParams {
    uint32_t N;    /* elements of D */
    uint32_t ne00; /* row length of A */
    uint32_t ne20; /* row length of D */
    uint32_t mode;
    float alpha, limit; /* unused by swiglu */
    uint32_t nb00, nb01, nb02, nb03;
    uint32_t nb10, nb11, nb12, nb13;
    uint32_t nb20, nb21, nb22, nb23;
    uint32_t ne21, ne22;
} MuyoGluParams;
int muyo_cuda_swiglu(const MuyoGluParams* p, const float* a, const float* b, float* d, void* stream);

/* ---- RoPE ---------------------------------------------------------------------------------------
 * Mirrors LlamaRopePushConstants (src/LlamaContracts.h:125-153) minus the set-rows fusion fields.
 * Replaces RopeExecute + rope_neox.comp / rope_norm (src/FullModel.cpp:179-212,
 * shaders/llama/rope_funcs.glsl:14-114). For row (i1, i2, i3): theta = pos[i2] * theta_scale^(i0/2)
 * (/ freq_factors[i0/2] if has_ff), YaRN-corrected when ext_factor != 0, negated if is_back; NEOX
 * pairs channels (j, j + n_dims/2), NORMAL pairs (2j, 2j+1); channels outside [n_offs, n_offs +
 * n_dims) are copied. Output element = d_offset + i1*nb11 + i2*nb12 + i3*nb13 + channel. */
#define MUYO_ROPE_NORMAL 0u
#define MUYO_ROPE_NEOX 2u
typedef struct MuyoRopeParams {
    uint32_t rope_mode;
    uint32_t nrows; /* ne01 * ne02 * ne03 */
    uint32_t n_dims;
    uint32_t n_offs;
    float freq_scale, freq_base, ext_factor, attn_factor;
    float corr_dims[2];
    float theta_scale;
    uint32_t has_ff;
    uint32_t is_back;
    uint32_t ne00, ne01, ne02;
    uint32_t nb01, nb02, nb03;
    uint32_t nb11, nb12, nb13;
    uint32_t a_offset, d_offset;
} MuyoRopeParams;
int muyo_cuda_rope(const MuyoRopeParams* p, const float* x, const int32_t* pos, const float* freq_factors, float* d,
                   void* stream);

/* ---- soft_max -----------------------------------------------------------------------------------
 * Mirrors LlamaSoftMaxPushConstants (src/LlamaContracts.h:255-274). Replaces SoftMaxExecute +
 * soft_max.comp (src/FullModel.cpp:331-349): per row, v = x*scale + slope*mask; D = exp(v - max) /
 * sum (+ exp(sink - max) in the sum if has_sinks). Rows: nrows_x of KX columns. */
typedef struct MuyoSoftMaxParams {
    uint32_t KX, KY;
    uint32_t ne00, ne01, ne02, ne12, ne13;
    uint32_t nb11, nb12, nb13;
    float scale, max_bias, m0, m1;
    uint32_t n_head_log2;
    uint32_t nrows_x;
    uint32_t has_sinks;
} MuyoSoftMaxParams;
int muyo_cuda_soft_max(const MuyoSoftMaxParams* p, const float* x, const float* mask, const float* sinks, float* d,
                       void* stream);

/* ---- argmax -------------------------------------------------------------------------------------
 * Mirrors LlamaGenericHeadPushConstants (src/LlamaContracts.h:224-232): KY rows of KX logits.
 * Replaces ArgmaxExecute + argmax.comp (src/FullModel.cpp:461-484) with the tie rule of the host's
 * greedy pick (src/Sampler.cpp:32-43): the FIRST index of the maximum. Large rows are split across
 * CTAs; the workspace (muyo_cuda_argmax_workspace_size bytes, any content) holds the partials. */
typedef struct MuyoGenericParams {
    uint32_t KX, KY;
    float param1, param2, param3, param4;
} MuyoGenericParams;
size_t muyo_cuda_argmax_workspace_size(const MuyoGenericParams* p);
int muyo_cuda_argmax(const MuyoGenericParams* p, const float* a, int32_t* d, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ---- copy (cpy_f32_f32) -------------------------------------------------------------------------
 * Mirrors copy.comp's unary head (src/FullModel.cpp:353-362) minus the fastdiv magic: element i of
 * the ne-element copy is read at A's coordinates of i (ne0x/nb0x) and written at D's coordinates
 * of i (ne1x/nb1x) plus d_offset. Replaces CopyValueColumnExecute's transposing V append
 * (src/FullModel.cpp:376-420), where the position travelled in misalign_offsets. */
typedef struct MuyoUnaryParams {
    uint32_t ne;
    uint32_t ne00, ne01, ne02, ne03, nb00, nb01, nb02, nb03;
    uint32_t ne10, ne11, ne12, ne13, nb10, nb11, nb12, nb13;
    uint32_t a_offset, d_offset;
} MuyoUnaryParams;
int muyo_cuda_copy_f32(const MuyoUnaryParams* p, const float* a, float* d, void* stream);

/* ---- decode attention over the KV cache ---------------------------------------------------------
 * Replaces the three-node scores GEMV -> soft_max -> value GEMV chain plus the K rope append and the
 * transposing V copy (src/FullModel.cpp:757-844; checks src/Attention.cpp:75-306 and
 * src/KvCache.cpp:94-430). One split-K flash-decoding kernel: the query heads of one KV head
 * (GQA group h / (heads/kv_heads), tools/reference_qwen2.py:133) share each K/V tile read.
 *
 * Cache layout (both K and V, row-major, no transpose): [kv_heads][max_seq][head_dim], element
 * type F32 (kv_dtype 0) or F16 (kv_dtype 1). The keys attended are 0 .. n_keys-1, where
 * n_keys = *pos + 1 when pos is non-NULL (device int32, read on the device so a captured graph
 * stays position-invariant) or p->n_keys otherwise. q: [heads][head_dim] F32, already rotated.
 * out: [heads][head_dim] F32. softmax scale p->scale (1/sqrt(head_dim) in the model). */
#define MUYO_KV_F32 0u
#define MUYO_KV_F16 1u
typedef struct MuyoAttentionParams {
    uint32_t heads, kv_heads, head_dim;
    uint32_t max_seq;
    uint32_t n_keys; /* used when pos == NULL */
    uint32_t kv_dtype;
    float scale;
} MuyoAttentionParams;
size_t muyo_cuda_attention_workspace_size(const MuyoAttentionParams* p);
int muyo_cuda_attention_decode(const MuyoAttentionParams* p, const float* q, const void* k_cache, const void* v_cache,
                               const int32_t* pos, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* KV append: rotate the new key (NEOX, theta = pos * base^(-2j/head_dim), in double precision as
 * tools/reference_qwen2.py:84-93) and store it and the new value at row *pos of each KV head,
 * rounded to the cache type. k, v: [kv_heads][head_dim] F32 (pre-rope key). Replaces k_rope with
 * dOffset = pos*headDim plus v_copy (src/FullModel.cpp:771-791). */
int muyo_cuda_kv_append(const MuyoAttentionParams* p, float rope_base, const float* k, const float* v, void* k_cache,
                        void* v_cache, const int32_t* pos, void* stream);

/* ---- fused Qwen2 decoder layer (one token) ------------------------------------------------------
 * One decoder layer of the reference's 18-node layer graph (src/FullModel.cpp:685-953) as five
 * fused kernels: [rms_norm + QKV GEMV + bias] -> [rope + KV append + split-K GQA attention
 * partials] -> [merge of the partials + o_proj GEMV + residual] -> [rms_norm + gate/up GEMV +
 * SwiGLU] -> [down GEMV + residual].
 * Weights F16 row-major [out][in] (GGUF [ne0 = in, ne1 = out]); biases and norms F32. wqkv is the
 * q, k and v projections stacked by rows ([q_dim + 2*kv_dim][hidden]) and bqkv their biases. */
typedef struct MuyoQwen2Config {
    uint32_t layers, hidden, ffn, heads, kv_heads, vocab, max_seq;
    float rms_eps, rope_base;
    uint32_t kv_dtype; /* MUYO_KV_F32 or MUYO_KV_F16 */
} MuyoQwen2Config;

typedef struct MuyoLayerWeights {
    const float* attn_norm;
    const void* wqkv;
    const float* bqkv;
    const void* wo;
    const float* ffn_norm;
    const void* wgate;
    const void* wup;
    const void* wdown;
} MuyoLayerWeights;

size_t muyo_cuda_layer_workspace_size(const MuyoQwen2Config* c);
/* x_in -> x_out (both [hidden] F32, may not alias); k_cache/v_cache are this layer's caches;
 * pos: device int32 position of the token. Weight matrices, norm weights, x_in and x_out must be
 * 16-byte aligned (MUYO_EINVAL otherwise); the workspace 256-byte aligned. */
int muyo_cuda_layer_step(const MuyoQwen2Config* c, const MuyoLayerWeights* w, void* k_cache, void* v_cache,
                         const int32_t* pos, const float* x_in, float* x_out, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ---- whole model (RunFullModel's engine) ---------------------------------------------------------
 * Replaces RunFullModel's graph build, weight upload and per-token feedToken/sampleNext loop
 * (src/FullModel.cpp:487-1291, header src/FullModel.h:34). The model owns its device weights, KV
 * cache and scratch (allocated once, in create/finalize - never per token). One decode step is
 * 5*layers+1 kernels captured in a CUDA graph (graphs of one and of eight steps, replayed in turn);
 * the position, the fed token and the greedy pick live in device memory, so a whole prompt +
 * generation is a loop of replays with no host round trip. */
typedef struct MuyoModel MuyoModel;
int muyo_model_create(const MuyoQwen2Config* c, int device, MuyoModel** out);
/* Upload one tensor by its GGUF name (src/FullModel.cpp:582-601), from host memory: F16 matrices
 * as binary16 bits, F32 vectors. output.weight may be omitted when tied to token_embd.weight. */
int muyo_model_set_tensor(MuyoModel* m, const char* name, const void* host, size_t bytes);
/* Load every tensor from a Qwen2 GGUF file (F16/F32 tensors, src/Gguf.cpp:337-348). */
int muyo_model_load_gguf(MuyoModel* m, const char* path);
/* Replaces ReadQwen2Config (src/FullModel.cpp:84-105): the qwen2.* dimensions, rms epsilon and
 * rope base of a GGUF file, and the vocabulary size as the length of tokenizer.ggml.tokens; the
 * cache capacity and KV type are the caller's. Reads the metadata only (no device work). */
int muyo_gguf_read_qwen2_config(const char* path, uint32_t max_seq, uint32_t kv_dtype, MuyoQwen2Config* out);
/* Check every tensor is present and build the step graphs. */
int muyo_model_finalize(MuyoModel* m, void* stream);
/* Empty the KV cache (positions restart at 0). */
int muyo_model_reset(MuyoModel* m, void* stream);
/* Feed prompt[0..n_prompt) then decode n_predict greedy ids (src/FullModel.cpp:1173-1208: every
 * fed and generated id passes one decode step, the last generated id included). Host buffers:
 * prompt is copied in, out_tokens (n_predict ids) copied back; blocks until done. Continues from
 * the current cache position (chat-style append), so call muyo_model_reset for a fresh sequence. */
int muyo_model_generate(MuyoModel* m, const int32_t* prompt, int n_prompt, int n_predict, int32_t* out_tokens,
                        void* stream);
/* Device-buffer variant (asynchronous on stream). */
int muyo_model_generate_device(MuyoModel* m, const int32_t* prompt_dev, int n_prompt, int n_predict,
                               int32_t* out_tokens_dev, void* stream);
/* One decode step for `token` at the current position; logits (vocab F32, device or host pointer,
 * may be NULL) and the greedy id (host, may be NULL) are returned. */
int muyo_model_step(MuyoModel* m, int32_t token, float* logits, int32_t* next_token, void* stream);
/* Current position (tokens in the cache). */
int muyo_model_position(const MuyoModel* m, int32_t* pos);
/* Device pointers of the model's buffers, for tests: "logits", "hidden", "k_cache", "v_cache". */
int muyo_model_buffer(MuyoModel* m, const char* name, void** ptr, size_t* bytes);
int muyo_model_destroy(MuyoModel* m);
/* Engine options: "engine" = 1 (the default) replays the per-phase kernels of muyo_cuda_layer_step
 * as a CUDA graph per decode step; 0 runs every decode step of a generate call in one persistent
 * cooperative kernel (a producer warp streams the weight rows of every phase into a shared-memory
 * ring ahead of the activation dependencies; consumer warps hand activations between phases as
 * {tag, value} words that the next phase polls; no grid barrier). Engine 0 takes greedy decoding
 * with head sizes 16..128 and shapes whose staging fits shared memory (MUYO_EUNSUPPORTED
 * otherwise, and while a sampler is set). Both compute the same arithmetic in F32; they differ
 * only in reduction order (last-bit differences, which an F16 cache can turn into one F16 ulp of a
 * key or value).
 * Graph-engine options (set before muyo_model_finalize; results are bit-identical either way):
 * "pdl" = 1 (default) launches each kernel with programmatic stream serialization, so it starts
 * while the previous kernel drains and waits on the device for that kernel's results; "prefetch" =
 * 1 (default) has each GEMV kernel stream the weights of the GEMV kernel two launches later into
 * L2; "smem_weights" = 1 (default) has the per-layer GEMV kernels copy their weight tile into shared
 * memory before waiting for the previous kernel (bounded wait; MUYO_ETIMEOUT if it expires). */
int muyo_model_set_option(MuyoModel* m, const char* key, int value);
/* Option "prefill" = 1 (default 0; allocates activations for one pass on first use): in
 * muyo_model_generate(_device), every prompt position but the last goes through the layers in
 * batched passes (muyo_cuda_mat_mul_f16's GEMM for the projections, a causal attention kernel
 * over the cache, on the tensor cores for an F16 cache), writing the same KV cache; the decode step then runs from the
 * prompt's last position. The reference feeds a prompt one position at a time (src/FullModel.cpp:
 * 1174-1181): results agree to float rounding, not bit for bit (the projections sum in another
 * order). No logits are formed for the batched positions. Option "prefill_tc" picks the projections'
 * GEMM (see muyo_cuda_mat_mul_f16): 0 the mma.sync kernel, 1 the tcgen05 kernel, 2 (default) per
 * GEMM: tcgen05 from 256 positions or for matrices of 4M weights and more. Option
 * "prefill_positions" (a multiple of 128 up to 1024, default 512; set before "prefill") is the
 * number of positions per pass; longer prompts take several passes. */

/* ---- batched F16 GEMM (the prefill projections) ---------------------------------------------------
 * y[t][n] = sum_k A[n][k] * x[t][k] for n < rows, t < tokens: ggml's mul_mm with src0 = A (F16,
 * [rows][ncols] row-major) and src1 = x (F32, tokens rows of stride_x), the batched counterpart of
 * muyo_cuda_mat_vec_f16 (the reference's shaders/llama/mul_mm.comp, which its engine never
 * dispatches). BIAS adds bias[n]; ACCUMULATE adds to y. x enters the tensor cores as two F16 halves
 * (hi = f16(x), lo = f16(x - hi)) with F32 accumulation: warp-level mma.sync on 64 x 64 tiles, or
 * with MUYO_MATMUL_TCGEN05 tcgen05.mma (tensor-memory accumulator, 128 x 64 tiles; slower at the
 * 0.5B layer's sizes while its tiles are fed by cp.async). ncols a multiple of 8; a, x and the
 * workspace 16-byte aligned. The kernels' waits are bounded (2 s); one that expired leaves y
 * unspecified (the model's prefill reports it as MUYO_ETIMEOUT). */
#define MUYO_MATMUL_BIAS 0x1u
#define MUYO_MATMUL_ACCUMULATE 0x2u
#define MUYO_MATMUL_TCGEN05 0x4u /* the tcgen05 kernel instead of the warp-level mma.sync one (the default) */
typedef struct MuyoMatMulParams {
    uint32_t ncols;    /* K */
    uint32_t rows;     /* N: output features */
    uint32_t tokens;   /* T: rows of x and y */
    uint32_t stride_x; /* 0 = ncols (a multiple of 4) */
    uint32_t stride_y; /* 0 = rows */
    uint32_t flags;
} MuyoMatMulParams;
size_t muyo_cuda_mat_mul_f16_workspace_size(const MuyoMatMulParams* p);
int muyo_cuda_mat_mul_f16(const MuyoMatMulParams* p, const void* a, const float* x, float* y, const float* bias,
                          void* workspace, size_t workspace_bytes, void* stream);

/* ---- row-sharded GEMV + cross-GPU greedy (multi-GPU LM head) --------------------------------------
 * One GPU's share of a row-sharded GEMV with the argmax folded into its epilogue: rows
 * [row_begin, row_begin + rows) of A ([rows][ncols] F16 local shard), d = A x, and the shard's
 * (max value, first global index) written to pair_out[0..1] as {float value, int32 index}.
 * The pairs of all ranks are exchanged (NCCL all-gather) and muyo_cuda_argmax_pairs picks the
 * first-index maximum over them. Workspace: muyo_cuda_argmax_workspace_size with KX = rows. */
int muyo_cuda_mat_vec_f16_argmax(const MuyoMatVecParams* p, const void* a, const float* b, float* d,
                                 uint32_t row_begin, void* pair_out, void* workspace, size_t workspace_bytes,
                                 void* stream);
int muyo_cuda_argmax_pairs(const void* pairs, uint32_t n_pairs, int32_t* d, void* stream);

/* ---- argmax with no workspace --------------------------------------------------------------------
 * No counterpart in the reference: an addition of this library for callers that cannot supply
 * device memory, either because allocating is off limits where they run (a memory budget already
 * carved up by a pool; a latency-critical loop that cannot take cudaMalloc's implicit device
 * synchronisation) or because they hold no device allocator (a thin FFI host that passes logits in
 * and reads an index back). Same contract and result as muyo_cuda_argmax; the partials live in a
 * static device array compiled into the library instead of a caller workspace, and the call
 * allocates nothing (no cudaMalloc, cudaFree or allocating library routine).
 *
 * Limit: KY * ceil(KX / 8192) partials must not exceed muyo_cuda_argmax_noalloc_max_pairs() (8192,
 * a 64 KB array per device): for example one row of up to 67,108,864 logits, or 431 rows of a
 * 151,936-entry vocabulary. Larger calls fail with MUYO_EINVAL and a message; nothing is launched.
 *
 * The first call on each device looks up the array's device address (cudaGetSymbolAddress, with
 * that device current) and caches it; make that first call before any stream capture. The cached
 * address belongs to the device's current context: do not call after a cudaDeviceReset.
 *
 * All calls on one device share the one array, so two calls that can run at the same time (on
 * different streams, or from different host threads without ordering) race on it and may return a
 * wrong index. Calls issued in order on a single stream are safe. */
size_t muyo_cuda_argmax_noalloc_max_pairs(void);
int muyo_cuda_argmax_noalloc(const MuyoGenericParams* p, const float* a, int32_t* d, void* stream);

/* ---- token sampler ------------------------------------------------------------------------------
 * Replaces Sampler::Sample (src/Sampler.cpp:10-98; parameters src/Sampler.h:14-22) on the device,
 * with the std::mt19937_64 stream kept in device memory (muyo_sampler_state_bytes bytes, 8-byte
 * aligned, seeded by muyo_sampler_seed as the engine's constructor seeds it). Same steps and order:
 * repetition penalty over the last repeat_last_n history tokens (negative: all; once per
 * occurrence), greedy when temperature <= 0 (first index of the maximum), else logits /= temperature,
 * top-k (top_k <= 0: the whole vocabulary), weights exp(double(l - l_max)), nucleus cut at top_p,
 * and a draw u = canonical double from the engine. logits is modified in place, as the reference
 * does. Equal logits are ordered by lower index (the reference's partial_sort leaves their order
 * unspecified). At most 4096 top-k candidates (MUYO_EUNSUPPORTED beyond). *token is a device int32. */
typedef struct MuyoSamplerParams {
    float temperature;
    int32_t top_k;
    float top_p;
    float repeat_penalty;
    int32_t repeat_last_n;
    uint32_t cluster_ctas; /* 0: automatic (16 CTAs where the device places them, else 8); 8 or 16 to force */
    uint64_t seed; /* used by muyo_model_set_sampler */
} MuyoSamplerParams;
size_t muyo_sampler_state_bytes(void);
int muyo_sampler_seed(void* state, uint64_t seed, void* stream);
int muyo_cuda_sample(const MuyoSamplerParams* p, float* logits, uint32_t vocab, const int32_t* history,
                     uint32_t hist_len, void* state, int32_t* token, void* stream);

/* Non-greedy decoding inside the model's step graph (RunFullModel's Sampler, src/FullModel.cpp:1058,
 * 1111-1116). Seeds a device engine with p->seed (synchronously on `stream`) and re-records the step
 * graph with a sampler node after the LM head. muyo_model_generate then samples every generated id
 * on the device: one draw per generated token, with every id in the cache (earlier turns, the prompt,
 * the ids generated so far) as the penalty history, and the engine's stream continuing across calls
 * as the reference's one Sampler does across turns. The logits buffer holds the penalised,
 * temperature-scaled logits afterwards, as the reference's mapped logits do. muyo_model_step is not
 * affected (it returns the logits and the greedy id; sample them with muyo_cuda_sample).
 * p == NULL, or temperature <= 0 with repeat_penalty == 1 (the reference's default), restores the
 * LM head's greedy pick. Needs the graph engine ("engine" 1); the persistent engine returns
 * MUYO_EUNSUPPORTED while a sampler is set. Limits as muyo_cuda_sample. */
int muyo_model_set_sampler(MuyoModel* m, const MuyoSamplerParams* p, void* stream);

/* ---- row-sharded GEMV fused with its all-gather over NVLink peer memory ---------------------------
 * No counterpart in the reference, which runs on one GPU: the multi-GPU form of its LM head +
 * greedy pick (src/FullModel.cpp:973-998, src/Sampler.cpp:32-43). `world` processes, one per GPU
 * of one node, each own a group. Set-up (allocates; not for the hot path):
 *   muyo_p2p_create   allocates this rank's buffer (a header and two slots of the full [rows_total]
 *                     F32 output) and writes its CUDA IPC handle (muyo_p2p_handle_bytes() bytes) to
 *                     handle_out;
 *   muyo_p2p_connect  opens every other rank's handle (handles: world of them, in rank order).
 * muyo_cuda_mat_vec_f16_allgather is a collective: every rank calls it, in the same order, with its
 * contiguous shard (rows [row_begin, row_begin + p->rows) of the full matrix; p->rows may be 0 when
 * there are more ranks than rows, and A is then not read). One kernel per GPU
 * computes the shard, stores it into every rank's output over NVLink, exchanges the shards'
 * (max, first index) pairs through peer memory as words tagged with the call's number (a pair that
 * arrives also says its rank's rows are in), and writes the greedy index to *token
 * (device int32) on every rank; the full output is then at muyo_p2p_output on every rank. Calls
 * alternate between the two output slots, so muyo_p2p_output (the slot of the latest call) changes
 * from call to call, and a peer that runs one call ahead writes the other slot. A peer reaches the
 * call after next (which rewrites this slot) only once this rank's next call has posted its pair, so
 * the output of a call stays intact until this rank's next call: read it on the same stream before.
 * The call count lives on the device, so calls may be captured in a CUDA graph and replayed (every
 * rank replaying the same calls): the n-th call since the group was created uses slot n & 1, and
 * muyo_p2p_output counts only the calls issued directly - after replays of a graph holding an odd
 * number of calls the caller picks the slot by the parity of its own total.
 * The wait for the peers is bounded (2 s): if a rank does not take part, the others finish with
 * token 0 and muyo_p2p_check (synchronising) reports MUYO_ETIMEOUT. The ranks' call counters then
 * disagree, so the group is dead: later calls return MUYO_ESTATE, and every rank must destroy its
 * group and create a new one. No multicast, no TMA: plain peer stores. */
typedef struct MuyoP2PGroup MuyoP2PGroup;
size_t muyo_p2p_handle_bytes(void);
int muyo_p2p_create(int world, int rank, uint32_t rows_total, MuyoP2PGroup** out, void* handle_out);
int muyo_p2p_connect(MuyoP2PGroup* g, const void* handles);
int muyo_cuda_mat_vec_f16_allgather(MuyoP2PGroup* g, const MuyoMatVecParams* p, const void* a, const float* b,
                                    uint32_t row_begin, int32_t* token, void* stream);
int muyo_p2p_output(MuyoP2PGroup* g, float** y);
int muyo_p2p_check(MuyoP2PGroup* g);
int muyo_p2p_destroy(MuyoP2PGroup* g);

#ifdef __cplusplus
}
#endif

#endif /* MUYO_CUDA_H */
