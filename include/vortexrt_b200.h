/*
 * vortexrt_b200.h -- C ABI of the B200 (sm_100a) backend for the Vortex-RT
 * Gemma 3 Q8_0 token loop.
 *
 * Every entry point returns 0 on success or a negative VRT_E_* code; the
 * message of the last failure on the calling thread is vrt_last_error().  No
 * C++ exception crosses this boundary.  Pointers named d_* are device
 * pointers, h_* host pointers.  `stream` is a cudaStream_t passed as void*
 * (NULL = the context's own stream).  Sizes are bytes unless named *_dim or
 * *_count.
 *
 * Each function cites the reference interface it replaces (paths inside the
 * Vortex-RT tree).  The reference's Vulkan layer (vulkan_context, buffer,
 * compute_pipeline) maps onto vrt_ctx_* / vrt_alloc / vrt_upload*; its
 * pipelines (Q8MatVecPipeline, ArgmaxPipeline) onto vrt_q8_* / vrt_argmax;
 * Gemma3Model onto vrt_model_*.
 */
#ifndef VORTEXRT_B200_H
#define VORTEXRT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VRT_API __attribute__((visibility("default")))

enum {
    VRT_OK = 0,
    VRT_E_INVALID = -1,   /* bad argument, shape, alignment or range        */
    VRT_E_CUDA = -2,      /* a CUDA runtime call failed                     */
    VRT_E_NOMEM = -3,     /* device or host allocation failed               */
    VRT_E_IO = -4,        /* file open / read / GGUF parse failure          */
    VRT_E_STATE = -5,     /* call order (positions, uninitialised model)    */
    VRT_E_NUMERIC = -6,   /* non-finite hidden state or invalid argmax      */
    VRT_E_TIMEOUT = -7,   /* a bounded device-side wait gave up             */
    VRT_E_UNSUPPORTED = -8
};

typedef struct vrt_ctx vrt_ctx;
typedef struct vrt_model vrt_model;

/* Result of an argmax: same layout as vortexrt::ArgmaxResult (include/vortexrt/argmax.hpp:12-17). */
typedef struct {
    uint32_t index;
    float value;
} vrt_argmax_result;

typedef struct {
    char name[256];
    int device;
    int sm_count;
    int cc_major, cc_minor;
    uint32_t warp_size;       /* reported where the reference reported subgroup_size */
    uint64_t global_mem_bytes;
    uint64_t l2_bytes;
} vrt_device_info;

/* ------------------------------------------------------------ runtime */

/* Thread-local message of the last failed call ("" if none). */
VRT_API const char* vrt_last_error(void);
VRT_API const char* vrt_version(void);

/* Open device `device` (-1 = VORTEXRT_DEVICE env var, else 0).
 * Replaces VulkanContext(device_selector) (src/vulkan_context.cpp:116-144). */
VRT_API int vrt_ctx_create(int device, vrt_ctx** out);
VRT_API int vrt_ctx_destroy(vrt_ctx* ctx);
/* Replaces VulkanContext::capabilities() (include/vortexrt/vulkan_context.hpp:56). */
VRT_API int vrt_ctx_info(vrt_ctx* ctx, vrt_device_info* out);
VRT_API int vrt_ctx_synchronize(vrt_ctx* ctx);
/* The context's stream (cudaStream_t). */
VRT_API void* vrt_ctx_stream(vrt_ctx* ctx);

/* Device allocation, 256-byte aligned, zero-filled, with 256 bytes of tail padding.
 * Replaces Buffer(ctx, size, usage, props) / ~Buffer (src/buffer.cpp:11-79). */
VRT_API int vrt_alloc(vrt_ctx* ctx, size_t bytes, void** d_out);
VRT_API int vrt_free(vrt_ctx* ctx, void* d_ptr);
/* Synchronous copies.  Replace Buffer::upload / Buffer::download (src/buffer.cpp:81-197). */
VRT_API int vrt_upload(vrt_ctx* ctx, void* d_dst, const void* h_src, size_t bytes);
VRT_API int vrt_download(vrt_ctx* ctx, void* h_dst, const void* d_src, size_t bytes);
/* Asynchronous copies on `stream` (host memory should be pinned for overlap). */
VRT_API int vrt_upload_async(vrt_ctx* ctx, void* d_dst, const void* h_src, size_t bytes, void* stream);
VRT_API int vrt_download_async(vrt_ctx* ctx, void* h_dst, const void* d_src, size_t bytes, void* stream);
VRT_API int vrt_host_alloc_pinned(size_t bytes, void** h_out);
VRT_API int vrt_host_free_pinned(void* h_ptr);

/* ---------------------------------------------- Q8_0 pipeline kernels
 * Weights are raw GGUF Q8_0 rows (34-byte blocks: fp16 scale + 32 int8) in a
 * device buffer of `weights_bytes`, at `weight_byte_offset` (4-byte aligned).
 * input_dim % 32 == 0.  Results are fp32.  Asynchronous on `stream`.
 * Accumulation: int8 weights x int16-quantised activation blocks, exact
 * integer block sums, fp32 across blocks. */

/* y[output_dim] = W x.  Replaces Q8MatVecPipeline::run (src/q8_matvec.cpp:801-930). */
VRT_API int vrt_q8_gemv(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes,
                        uint64_t weight_byte_offset, const float* d_x, float* d_y,
                        uint32_t input_dim, uint32_t output_dim, void* stream);

/* `count` (1..8) mat-vecs sharing x; outputs packed back to back in d_y
 * (matrix i at element sum(output_dims[0..i))).  Replaces
 * Q8MatVecPipeline::run_staged_pair / run_staged_triplet (src/q8_matvec.cpp:2007-2890). */
VRT_API int vrt_q8_gemv_multi(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes,
                              const uint64_t* weight_byte_offsets, const uint32_t* output_dims,
                              uint32_t count, const float* d_x, float* d_y, uint32_t input_dim,
                              void* stream);

/* y = W_down (gelu_tanh(W_gate x) * (W_up x)).  d_workspace holds 2*ffn_dim floats.
 * Replaces Q8MatVecPipeline::run_staged_ffn (src/q8_matvec.cpp:1360-2004). */
VRT_API int vrt_q8_ffn(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes,
                       uint64_t gate_off, uint64_t up_off, uint64_t down_off, const float* d_x,
                       float* d_workspace, float* d_y, uint32_t input_dim, uint32_t ffn_dim,
                       uint32_t output_dim, void* stream);

/* The fused FFN above for callers that cannot allocate device memory: no
 * context and no workspace argument; runs on the current device.  No
 * counterpart in the reference.  The gate/up intermediate lives in a
 * library-owned device array of 2 * 32768 floats (256 KB on every GPU that
 * loads the library, held until exit), so ffn_dim <= 32768 (larger sizes
 * return VRT_E_INVALID) and nothing is ever allocated.  The first call on a
 * device looks up that array's device address (cudaGetSymbolAddress); make
 * that first call before any stream capture.  That set-up is kept for the
 * life of the process and is not redone after cudaDeviceReset: do not call
 * this after resetting a device that it has run on.  All calls share the one
 * array: calls that overlap on the GPU (other streams, other threads) race on
 * it.  `stream` NULL = the CUDA default stream. */
VRT_API int vrt_q8_ffn_static(const void* d_weights, uint64_t weights_bytes, uint64_t gate_off,
                              uint64_t up_off, uint64_t down_off, const float* d_x, float* d_y,
                              uint32_t input_dim, uint32_t ffn_dim, uint32_t output_dim, void* stream);

/* gate[i] = gelu_tanh(gate[i]) * up[i].  Replaces shaders/gelu_mul.comp. */
VRT_API int vrt_gelu_mul(vrt_ctx* ctx, float* d_gate, const float* d_up, uint32_t count, void* stream);

/* argmax over count floats: ties -> lower index, NaN never wins; all-NaN gives
 * {0xffffffff, -inf}.  Replaces ArgmaxPipeline::run (src/argmax.cpp:503-567). */
VRT_API int vrt_argmax(vrt_ctx* ctx, const float* d_x, uint32_t count, vrt_argmax_result* d_out,
                       void* stream);

/* Tied LM head fused with argmax: the logits never reach memory unless
 * d_logits != NULL.  Replaces run_q8_matvec_to_output + ArgmaxPipeline::run
 * (src/gemma3.cpp:1146-1185). */
VRT_API int vrt_lm_head_argmax(vrt_ctx* ctx, const void* d_weights, uint64_t weights_bytes,
                               uint64_t weight_byte_offset, const float* d_x, uint32_t input_dim,
                               uint32_t vocab, float* d_logits, vrt_argmax_result* d_out,
                               void* stream);

/* Device error word of the pipeline entry points above (bit 0: a bounded
 * wait of the staged mat-vec kernel for its own bulk copy gave up, after
 * about a second; that call's outputs are then undefined), read and cleared.
 * ctx != NULL: the context's calls (its stream is synchronised first);
 * ctx == NULL: vrt_q8_ffn_static's calls on the current device (synchronise
 * the stream they ran on first).  No counterpart in the reference, whose
 * shaders have no waits. */
VRT_API int vrt_pipeline_status(vrt_ctx* ctx, uint32_t* h_status);

/* --------------------------------------- packed (Q8T) fast path
 * The model's own weight layout, exposed for callers that keep a matrix
 * resident and call it many times: rows of 16 x 128-column tiles, each tile's
 * bytes in the order one warp consumes them (same 34 bytes per 32 weights as
 * GGUF).  cols % 128 == 0.  Tiled mat-vecs stream the weights with bulk
 * copies through shared memory.  No reference counterpart: these are the
 * kernels behind vrt_model_* made callable on their own. */

VRT_API uint64_t vrt_q8t_bytes(uint32_t rows, uint32_t cols);
/* Repack `rows` raw Q8_0 rows at byte `offset` of d_raw into d_packed (vrt_q8t_bytes(rows, cols) bytes). */
VRT_API int vrt_q8t_pack(vrt_ctx* ctx, const void* d_raw, uint64_t raw_bytes, uint64_t offset, uint32_t rows,
                         uint32_t cols, void* d_packed, void* stream);
/* Interleave gate and up matrices (ffn rows each) into one packed pair (vrt_q8t_bytes(2*ffn, cols)). */
VRT_API int vrt_q8t_pack_pair(vrt_ctx* ctx, const void* d_raw, uint64_t raw_bytes, uint64_t gate_offset,
                              uint64_t up_offset, uint32_t ffn, uint32_t cols, void* d_packed, void* stream);
/* y = W x with W packed. */
VRT_API int vrt_q8t_gemv(vrt_ctx* ctx, const void* d_packed, uint32_t rows, uint32_t cols, const float* d_x,
                         float* d_y, void* stream);
/* act = gelu_tanh(W_gate x) * (W_up x), one kernel over a packed pair. */
VRT_API int vrt_q8t_gate_up(vrt_ctx* ctx, const void* d_packed_pair, uint32_t ffn, uint32_t cols,
                            const float* d_x, float* d_act, void* stream);
/* Fused FFN over packed weights: two kernels (gate/up + gelu, down). */
VRT_API int vrt_q8t_ffn(vrt_ctx* ctx, const void* d_gate_up, const void* d_down, uint32_t input_dim,
                        uint32_t ffn_dim, uint32_t output_dim, const float* d_x, float* d_act, float* d_y,
                        void* stream);
/* Tensor-core (tcgen05) GEMM over a packed matrix: d_y[m][rows] = d_x[m][cols] . W^T
 * for m activation rows (prompt tokens or batched sequences), rows % 128 == 0.
 * Operands are split into fp16 hi + lo terms (three MMAs, fp32 accumulation:
 * ~1e-7 relative error).  Synchronous; uses a context scratch of
 * 4*m*cols bytes.  No reference counterpart: the reference runs every prompt
 * token through the mat-vec path (src/gemma3.cpp:2080-2149). */
VRT_API int vrt_q8t_gemm(vrt_ctx* ctx, const void* d_packed, uint32_t rows, uint32_t cols, const float* d_x,
                         uint32_t m, float* d_y, void* stream);
/* Gate/up pair form (d_packed_pair from vrt_q8t_pack_pair, ffn % 64 == 0):
 * d_act[m][ffn] = gelu_tanh(gate) * up, the batched run_staged_ffn first half
 * (src/q8_matvec.cpp:1360-2004 per token). */
VRT_API int vrt_q8t_gemm_gelu(vrt_ctx* ctx, const void* d_packed_pair, uint32_t ffn, uint32_t cols,
                              const float* d_x, uint32_t m, float* d_act, void* stream);
/* Few-row form on the integer tensor cores (tcgen05 kind::i8), 1 <= m <= 32:
 * the packed matrix is first copied into the Q8M layout (128 x 128 int8
 * operand tiles in the MMA's swizzled order + fp16 block scales; same byte
 * count as the packed matrix), the activation rows are quantised per
 * 32-block to int16 (split into two int8 halves), each Q8_0 block is one
 * exact int32 MMA, and the block scales are applied in fp32 afterwards.
 * Synchronous; uses the context scratch (about 2*m*cols bytes plus split-K
 * partials), like vrt_q8t_gemm.  The gelu form takes a Q8M copy of a
 * vrt_q8t_pack_pair matrix. */
VRT_API int vrt_q8t_to_q8m(vrt_ctx* ctx, const void* d_packed, uint32_t rows, uint32_t cols, void* d_out,
                           void* stream);
VRT_API int vrt_q8m_gemm(vrt_ctx* ctx, const void* d_q8m, uint32_t rows, uint32_t cols, const float* d_x,
                         uint32_t m, float* d_y, void* stream);
VRT_API int vrt_q8m_gemm_gelu(vrt_ctx* ctx, const void* d_q8m_pair, uint32_t ffn, uint32_t cols,
                              const float* d_x, uint32_t m, float* d_act, void* stream);
/* LM head + argmax over a packed vocab matrix (logits written when d_logits != NULL). */
VRT_API int vrt_q8t_lm_head_argmax(vrt_ctx* ctx, const void* d_packed, uint32_t vocab, uint32_t cols,
                                   const float* d_x, float* d_logits, vrt_argmax_result* d_out, void* stream);

/* ------------------------------------------------------------ model */

typedef struct {
    uint32_t context_length, embedding_length, block_count, feed_forward_length;
    uint32_t head_count, head_count_kv, head_dim, value_dim, vocab_size, sliding_window;
    float rms_epsilon, global_rope_base, local_rope_base;
} vrt_gemma3_config; /* = vortexrt::Gemma3Config (include/vortexrt/gemma3.hpp:19-33) */

typedef struct {
    uint32_t max_positions; /* KV/rope capacity; 0 = min(context_length, 8192) */
    int tp_rank;            /* tensor-parallel rank (0 when tp_world <= 1)      */
    int tp_world;           /* tensor-parallel width (0/1 = single GPU)         */
    const void* nccl_id;    /* ncclUniqueId bytes when tp_world > 1             */
    int use_graph;          /* capture the decode step in a CUDA graph          */
    int use_pdl;            /* programmatic dependent launch between kernels    */
    int tp_exchange;        /* VRT_TP_PEER (default) or VRT_TP_NCCL             */
    uint32_t tp_wait_ms;    /* bound of one wait on a peer; 0 = 10000 ms        */
    uint32_t prefill_chunk; /* prompt tokens per batched (tensor-core) prefill
                               pass; 0 = 2048; 1 = token by token through the
                               decode step, the reference's method            */
    int step_mode;          /* VRT_STEP_LAUNCHES (default) or VRT_STEP_PERSISTENT */
} vrt_model_options;

/* How one decode step runs on the GPU.  VRT_STEP_PERSISTENT: one cooperative
 * kernel per token (one CTA per SM) streams every layer's weights without
 * pausing at op boundaries and passes activations between CTAs as tagged
 * words, with no grid barrier and no launch between ops.  VRT_STEP_LAUNCHES:
 * one kernel per op (5 per layer), chained by programmatic dependent launch.
 * The persistent form needs a single GPU or tp_exchange = VRT_TP_PEER; other
 * cases use the launch chain.  Both give the same tokens up to fp32 addition
 * order. */
enum { VRT_STEP_PERSISTENT = 0, VRT_STEP_LAUNCHES = 1 };

/* How the partial sums of the row-parallel projections (attention output,
 * FFN down) and the per-rank argmax keys are combined under tensor
 * parallelism.  VRT_TP_PEER: the consuming kernel pushes its rank's partials
 * into the peers' memory (CUDA IPC over NVLink) and sums all ranks' partials
 * in rank order inside its prologue -- no separate collective kernel.
 * VRT_TP_NCCL: an NCCL all-reduce after each row-parallel projection (the
 * plain form, kept for comparison).  Both give the same sums up to fp32
 * addition order. */
enum { VRT_TP_PEER = 0, VRT_TP_NCCL = 1 };

/* Defaults: max_positions 0, single GPU, use_graph = 1, use_pdl = 1,
 * tp_exchange = VRT_TP_PEER, tp_wait_ms = 0, prefill_chunk = 0,
 * step_mode = VRT_STEP_LAUNCHES.  Prompts of
 * two or more tokens are prefilled in batched tensor-core passes (under
 * tensor parallelism with NCCL sums of the row-parallel partials) unless
 * tracing is on or prefill_chunk = 1; then they go token by token. */
VRT_API void vrt_model_options_default(vrt_model_options* o);

/* Load a Gemma 3 Q8_0 GGUF: weights repacked into the device arena, norms,
 * rope tables and KV cache allocated.  Replaces the Gemma3Model constructor
 * (src/gemma3.cpp:72-654); lifts its one-KV-head and 4 GiB limits. */
VRT_API int vrt_model_load(vrt_ctx* ctx, const char* gguf_path, const vrt_model_options* opts,
                           vrt_model** out);

/* Build the seeded synthetic model of the given shape directly in device
 * memory (the generator of synth_gguf.py, bit-identical to loading the file
 * it writes).  For benchmarks of shapes too large to write as files. */
VRT_API int vrt_model_create_synthetic(vrt_ctx* ctx, const vrt_gemma3_config* cfg, uint64_t seed,
                                       const vrt_model_options* opts, vrt_model** out);
VRT_API int vrt_model_destroy(vrt_model* m);
VRT_API int vrt_model_config(vrt_model* m, vrt_gemma3_config* out);

/* Gemma3Model::reset_cache (src/gemma3.cpp:1454-1460). */
VRT_API int vrt_model_reset(vrt_model* m);

/* Gemma3Model::decode_token (src/gemma3.cpp:1462-1882).  position must equal
 * the next position.  top_k == 0 skips the LM head; 1 = fused LM head +
 * argmax; >1 = full logits, top-k by value (ties -> lower id).  h_hidden
 * (optional) receives the final normed hidden state (embedding_length
 * floats); h_ids/h_logits receive min(top_k, vocab) entries.  Under tensor
 * parallelism every rank makes the same call; with top_k > 1 the ranks'
 * logits shards are all-gathered and every rank returns the same top-k. */
VRT_API int vrt_decode_step(vrt_model* m, uint32_t token, uint32_t position, uint32_t top_k,
                            float* h_hidden, uint32_t* h_ids, float* h_logits);

/* Full-vocabulary logits of the last decode step into h_logits (vocab
 * floats).  Under tensor parallelism it gathers every rank's shard: all ranks
 * must call it together. */
VRT_API int vrt_model_logits(vrt_model* m, float* h_logits);

/* Gemma3Model::generate_greedy_tokens (src/gemma3.cpp:2080-2149): token-by-token
 * prefill, greedy decode until max_new tokens or EOS.  Runs on the device with
 * no host round trip per token; h_out receives *h_count <= max_new ids. */
VRT_API int vrt_generate_greedy(vrt_model* m, const uint32_t* h_prompt, uint32_t prompt_count,
                                uint32_t max_new, uint32_t* h_out, uint32_t* h_count);

/* Device-resident continuation for benchmarks: runs `steps` greedy decode steps
 * from the current state, the i-th generated id written to d_out_ids[i] when
 * non-NULL.  No host synchronisation.  Needs a prefill or a decode step with
 * top_k > 0 first (VRT_E_STATE otherwise): the step state then holds a greedy
 * id to continue from. */
VRT_API int vrt_decode_steps_async(vrt_model* m, uint32_t steps, uint32_t* d_out_ids, void* stream);

/* Prefill helper: feeds prompt tokens through the decode step without the LM
 * head (the reference's top_k = 0 prompt steps) except the last one.  After it
 * the model holds the argmax of the last prompt token as its next input. */
VRT_API int vrt_prefill(vrt_model* m, const uint32_t* h_prompt, uint32_t prompt_count);

/* Greedy token that the next vrt_decode_steps_async step will consume. */
VRT_API int vrt_model_next_token(vrt_model* m, uint32_t* h_token, uint32_t* h_position);

/* Number of kernels one decode step launches (graph nodes), for reporting. */
VRT_API int vrt_model_step_kernels(vrt_model* m, uint32_t* out);

/* Device error word (bounded waits that gave up, invalid tokens) and clear it. */
VRT_API int vrt_model_device_status(vrt_model* m, uint32_t* h_status);

/* Per-layer residual trace of the last decode step (block_count x d floats),
 * for debugging against the CPU oracle.  Enabled by vrt_model_set_trace(m, 1). */
VRT_API int vrt_model_set_trace(vrt_model* m, int enabled);
VRT_API int vrt_model_trace(vrt_model* m, float* h_out);

/* Benchmark helper: average device time of one of the decode step's
 * mat-vec launches run alone (0 qkv, 1 o-proj, 2 gate/up, 3 down, 4 LM head
 * of `layer`), and its algorithmic bytes (weights + vectors once).  Clobbers
 * activations; call vrt_model_reset before decoding again. */
VRT_API int vrt_model_time_kernel(vrt_model* m, uint32_t layer, uint32_t which, uint32_t iters,
                                  float* ms_per_launch, uint64_t* algorithmic_bytes);

/* ---------------------------------------------------------- batched decode
 * Independent sequences decoded together (no reference counterpart: the
 * reference decodes one sequence, src/gemma3.cpp:1462-1882), on one GPU or a
 * tensor-parallel model (every rank holds every sequence; all ranks make the
 * same calls).  Each sequence has its own KV cache; a step decodes one greedy
 * token for each of the first `count` sequences, with the projections and the
 * tied LM head as tensor-core GEMMs of `count` rows (integer tensor cores up to
 * 32 rows, fp16 above).  Per sequence the results match decoding it alone
 * within the north-star tolerance. */
typedef struct vrt_batch vrt_batch;
/* max_positions <= the model's positions; keep_logits != 0 keeps the last
 * step's full logits per sequence (max_seqs * vocab floats) for checking.
 * The first batch of a model also makes the model's Q8M weight copy for the
 * integer GEMM (the size of the Q8_0 weights again; skipped, with the fp16
 * GEMMs used instead, when it does not fit). */
VRT_API int vrt_batch_create(vrt_model* m, uint32_t max_seqs, uint32_t max_positions, int keep_logits,
                             vrt_batch** out);
VRT_API int vrt_batch_destroy(vrt_batch* b);
/* Prefill sequence `seq` (batched tensor-core prefill into its cache); emits its
 * first greedy id and sets its position to n. */
VRT_API int vrt_batch_prefill(vrt_batch* b, uint32_t seq, const uint32_t* h_prompt, uint32_t n);
/* `steps` greedy steps of sequences [0, count), queued on the model stream. */
VRT_API int vrt_batch_decode_steps(vrt_batch* b, uint32_t count, uint32_t steps);
/* Ids generated for `seq` so far (first min(count, cap) into h_ids), its count
 * and next position.  Synchronises with the model stream. */
VRT_API int vrt_batch_read(vrt_batch* b, uint32_t seq, uint32_t* h_ids, uint32_t cap, uint32_t* h_count,
                           uint32_t* h_position);
/* The latest generated id of each of the first `count` sequences (their next
 * input tokens) into h_ids; synchronises with the model stream. */
VRT_API int vrt_batch_last_ids(vrt_batch* b, uint32_t count, uint32_t* h_ids);
/* Last step's logits of `seq` (vocab floats; needs keep_logits). */
VRT_API int vrt_batch_logits(vrt_batch* b, uint32_t seq, float* h_logits);

/* ------------------------------------------------------ tokenizer (host)
 * The GGUF vocabulary's tokenizer with the reference's rules
 * (src/gemma3.cpp:289-454 index, 1895-2062 tokenize, 1237-1299 pieces); no
 * GPU involved. */
typedef struct vrt_tokenizer vrt_tokenizer;
VRT_API int vrt_tokenizer_open(const char* gguf_path, vrt_tokenizer** out);
VRT_API void vrt_tokenizer_close(vrt_tokenizer* t);
/* Gemma3Model::tokenize: *n receives the id count (ids beyond cap are dropped). */
VRT_API int vrt_tokenize(vrt_tokenizer* t, const char* text, int add_bos, uint32_t* out, size_t cap, size_t* n);
/* token_piece (decoded = 0) or decode_piece (decoded = 1), NUL-terminated into out[cap]. */
VRT_API int vrt_token_piece(vrt_tokenizer* t, uint32_t id, int decoded, char* out, size_t cap, size_t* n);

/* ------------------------------------------------- tensor parallelism
 * Rank `rank` of `world` holds query heads [q_head0, q_head0+q_heads), KV heads
 * [kv_head0, ...), FFN rows [ffn0, ffn0+ffn) of gate/up (= K columns of down),
 * and vocab rows [vocab0, vocab0+vocab) of the LM head.  o-proj takes the K
 * columns of its query heads.  No reference counterpart (the reference is
 * single-device). */
typedef struct {
    uint32_t q_head0, q_heads, kv_head0, kv_heads, ffn0, ffn, vocab0, vocab;
} vrt_tp_shard;
VRT_API int vrt_tp_plan(const vrt_gemma3_config* cfg, int world, int rank, vrt_tp_shard* out);

/* NCCL unique id for tensor parallelism (128 bytes). */
VRT_API int vrt_tp_unique_id(void* h_out128);

#ifdef __cplusplus
}
#endif

#endif /* VORTEXRT_B200_H */
