/*
 * nvkv.h -- C ABI of the B200 (sm_100a) attention hot path for nanovllm_rs.
 *
 * One shared library, libnvkv.so, exports every function below with C
 * linkage.  The signatures carry plain device pointers, sizes and a
 * cudaStream_t only (no framework tensor types), so a Rust `-sys` crate,
 * ctypes or any C caller can bind them directly.
 *
 * Conventions (shared by every entry point):
 *  - Return value: NVKV_OK (0) on success, a negative NVKV_ERR_* code
 *    otherwise.  Arguments are validated on the host before anything is
 *    launched; on error nothing is launched and nvkv_last_error() returns a
 *    message for the calling thread.  No C++ exception crosses the ABI.
 *  - Every buffer belongs to the caller.  Kernels are enqueued on `stream`
 *    and read/write the buffers asynchronously; inputs must stay alive until
 *    the stream passes the launch (the ownership model of the reference's
 *    candle custom ops, nanovllm_rs/src/layers/kv_cache.rs:130-151).
 *  - The CUDA device current on the calling thread must own every pointer
 *    (the reference binds one device per rank thread,
 *    nanovllm_rs/src/layers/dist_util.rs:50-53).
 *  - dtype is NVKV_DTYPE_BF16 or NVKV_DTYPE_F16 (the two dtypes the
 *    reference's store kernel and flash-attn accept, kv_cache.rs:154-158).
 *  - Device-side bounds checks (slot >= number of cache rows, block id >=
 *    number of pages, position >= max_position) skip the offending access and
 *    record an error code that nvkv_device_error() reports.
 */
#ifndef NVKV_H_
#define NVKV_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* nvkv_stream_t; /* == cudaStream_t */

#define NVKV_OK 0
#define NVKV_ERR_INVALID_ARG (-1)   /* bad shape / null pointer / size       */
#define NVKV_ERR_UNSUPPORTED (-2)   /* dtype, head_dim, page size, group     */
#define NVKV_ERR_ALIGNMENT (-3)     /* pointer or stride not 16-byte aligned */
#define NVKV_ERR_CUDA (-4)          /* a CUDA runtime/driver call failed     */
#define NVKV_ERR_WORKSPACE (-5)     /* workspace missing or too small        */
#define NVKV_ERR_DEVICE (-6)        /* a kernel recorded a bounds violation  */

#define NVKV_DTYPE_F16 0
#define NVKV_DTYPE_BF16 1
#define NVKV_DTYPE_F32 2 /* logits of nvkv_sample only */

/* Device-side error codes reported by nvkv_device_error(). */
#define NVKV_DEVERR_NONE 0
#define NVKV_DEVERR_SLOT_RANGE 1      /* slot_mapping[t] >= num_slots         */
#define NVKV_DEVERR_BLOCK_RANGE 2     /* block_tables entry >= num_blocks     */
#define NVKV_DEVERR_POSITION_RANGE 3  /* positions[t] outside [0, max_pos)    */
#define NVKV_DEVERR_SEQLEN 4          /* q_len > k_len or lengths > maxima    */

/* Library version (major*10000 + minor*100 + patch). */
int nvkv_version(void);

/* Message for the last failing call on this thread ("" if none). */
const char* nvkv_last_error(void);

/* Reads (and if `clear` != 0 resets) the current device's error word that
 * kernels set when a bounds check fails.  Synchronises the device.  */
int nvkv_device_error(int* code, int clear);

/* ------------------------------------------------------------------------
 * Kernel 1: KV-cache scatter.
 * Replaces: nanovllm_rs/src/layers/kv_cache.rs:168-190 (store_kv_cache) and
 *           kv_cache.rs:102-161 (StoreKvCache::cuda_fwd launching the NVRTC
 *           kernels of kv_cache.rs:9-38).
 *
 * k_cache[slot_mapping[t] * row_elems + i] = key[t * key_stride + i]
 * v_cache[slot_mapping[t] * row_elems + i] = value[t * value_stride + i]
 * for t < num_tokens, i < row_elems (= num_kv_heads * head_dim), skipping
 * tokens whose slot is negative (the reference's padding/warm-up rule,
 * kv_cache.rs:19-20).  Caches are [num_slots, row_elems] =
 * [num_blocks * block_size, num_kv_heads * head_dim].  key/value may be
 * strided views (e.g. the K and V slices of a fused qkv buffer), so no
 * contiguous copy is needed first (the reference's force_contiguous,
 * kv_cache.rs:175-186).  One launch writes both caches.  Bit-exact copy.
 * ---------------------------------------------------------------------- */
int nvkv_store_kvcache(const void* key, const void* value, void* k_cache, void* v_cache,
                       const int64_t* slot_mapping, int64_t num_tokens, int64_t row_elems,
                       int64_t key_stride, int64_t value_stride, int64_t num_slots,
                       int dtype, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Kernel 4: fused qk-RMSNorm + RoPE prologue (optionally fused with kernel 1).
 * Replaces: nanovllm_rs/src/models/qwen3.rs:128-141 (split_qkv, per-head
 *           q_norm/k_norm, rotary_emb.forward), i.e. layers/layernorm.rs:18-25
 *           and layers/rotary_embedding.rs:11-70.
 *
 * qkv: [num_tokens, (Hq + 2*Hkv) * head_dim] with row stride `qkv_stride`
 *      elements (the output of the fused QKV projection).
 * For each token t and head h:
 *   x  = q or k head row;  x' = dtype(x * rsqrt(mean(x^2) + eps)) * w
 *        (rounded to dtype after the normalise and after the weight multiply,
 *        like the reference); skipped when q_norm_w == k_norm_w == NULL.
 *   RoPE (NeoX half split) at positions[t] with inv_freq_i =
 *        1 / exp((2i/D) * ln(theta)), cos/sin computed in f32 and rounded to
 *        dtype before use, each product/sum rounded to dtype.
 * Outputs: q_out [T, Hq, D] (required); k_out/v_out [T, Hkv, D] (optional,
 * NULL to skip; needed only when attention runs without a KV cache).  When
 * k_cache/v_cache/slot_mapping are non-NULL the rotated K and the V rows are
 * also scattered into the caches exactly as nvkv_store_kvcache would.
 * positions must lie in [0, max_position) (the reference's cos/sin table
 * has max_position rows, rotary_embedding.rs:38-49).  head_dim must be 128.
 * q_norm_w/k_norm_w are [head_dim] in `dtype`.
 * ---------------------------------------------------------------------- */
int nvkv_qknorm_rope(const void* qkv, int64_t qkv_stride, int64_t num_tokens, int num_q_heads,
                     int num_kv_heads, int head_dim, const int64_t* positions,
                     const void* q_norm_w, const void* k_norm_w, float eps, float rope_theta,
                     int64_t max_position, void* q_out, void* k_out, void* v_out, void* k_cache,
                     void* v_cache, const int64_t* slot_mapping, int64_t num_slots, int dtype,
                     nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Kernels 2 + 3: varlen (paged) causal attention with GQA.
 * Replaces: nanovllm_rs/src/layers/attention.rs:37-75 (the calls to
 *           candle_flash_attn::flash_attn_varlen_paged_windowed with
 *           window (None, Some(0)) and flash_attn_varlen(causal=true)).
 *
 * q:   [num_q_tokens, Hq, D] with token stride q_stride (elements); head
 *      stride D.
 * out: [num_q_tokens, Hq, D] contiguous.
 * Device-side checks (the metadata lives on the device, so the host cannot
 * see it): a sequence whose query rows cu_seqlens_q[b] .. cu_seqlens_q[b+1]
 * reach past num_q_tokens, whose k_len exceeds max_seqlen_k, or (q_len > 1)
 * whose k_len is below its q_len is skipped -- none of its q rows are read,
 * none of its out rows written, no block-table entry beyond max_seqlen_k keys
 * read -- and NVKV_DEVERR_SEQLEN is recorded for nvkv_device_error().  A page id >=
 * num_blocks reads page 0 instead and records NVKV_DEVERR_BLOCK_RANGE.
 * Paged (block_tables != NULL): k_cache/v_cache are [num_blocks, page_size,
 *      Hkv, D]; key j of sequence b lives in page block_tables[b *
 *      block_table_stride + j / page_size], row j % page_size.
 * Contiguous (block_tables == NULL): k_cache/v_cache are [Tk, Hkv, D] and
 *      sequence b owns rows cu_seqlens_k[b] .. cu_seqlens_k[b+1]; num_blocks
 *      is then the row count Tk and page_size is ignored.
 * kv_stride: elements between consecutive rows (slots / tokens) of k_cache
 *      and v_cache; 0 means Hkv * D (dense).  A multiple of 8, so the K/V
 *      slices of a fused qkv buffer can be attended in place.
 * cu_seqlens_q/k: [num_seqs + 1] uint32 prefix sums (device memory).
 * Query i of sequence b (q_len = cu_q[b+1]-cu_q[b], k_len likewise) sees key
 * j iff j <= i + k_len - q_len when causal != 0 (all keys otherwise).
 * Sequences with q_len == 1 run on the split-KV paged decode kernel
 * (TMA-staged K/V, warp-shuffle softmax, LSE combine); the others run on the
 * tcgen05 prefill kernel.  max_seqlen_q/k bound the per-sequence lengths.
 * D must be 128; Hq % Hkv == 0 with Hq/Hkv <= 16; page_size a multiple of
 * 128.  `workspace` must hold nvkv_paged_attention_workspace_size() bytes
 * (16-byte aligned); it may be NULL when that size is 0.  It holds the
 * split-KV scratch and, when max_seqlen_q > 1, the prefill work plan (a
 * sort of the q_len > 1 sequences by q-tile count, about 4 * (num_seqs +
 * max_seqlen_q / 128) bytes), rebuilt by every call.
 * ---------------------------------------------------------------------- */
int nvkv_paged_attention_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads,
                                        int head_dim, int max_seqlen_q, int max_seqlen_k,
                                        size_t* bytes);

int nvkv_paged_attention(const void* q, int64_t q_stride, int64_t num_q_tokens,
                         const void* k_cache, const void* v_cache, int64_t num_blocks,
                         int64_t kv_stride, void* out,
                         const uint32_t* cu_seqlens_q, const uint32_t* cu_seqlens_k,
                         const uint32_t* block_tables, int64_t block_table_stride, int num_seqs,
                         int max_seqlen_q, int max_seqlen_k, int num_q_heads, int num_kv_heads,
                         int head_dim, int page_size, float softmax_scale, int causal,
                         void* workspace, size_t workspace_bytes, int dtype,
                         nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * FP8 (e4m3) KV pool: an optional pool format at half the bytes.
 * No counterpart in the reference, whose pool is in the model dtype
 * (nanovllm_rs/src/engine/model_runner.rs:286-303); it stands beside the
 * store of kv_cache.rs:168-190 and the attention of attention.rs:37-75.
 *
 * Layout: k_cache / v_cache [num_blocks, page_size, Hkv, 128] one-byte e4m3
 * codes (the dtype pool's slot addressing); k_scale / v_scale
 * [num_blocks, Hkv, page_size] f32, one scale per (slot, kv head) row:
 *   scale = amax / 448, code = e4m3_rn_satfinite(x * (448 / amax)),
 *   value = code * scale   (amax = max |x| over the row's 128 values; a row
 *   of zeros gets scale 0).  Division and product are f32, rounded to nearest.
 *
 * nvkv_store_kvcache_fp8: quantises rows t < num_tokens of key/value
 * ([T, Hkv, 128] bf16/f16 with token strides key_stride / value_stride
 * elements, a multiple of 4; rows 8-byte aligned) into slot slot_mapping[t]
 * (negative: skipped; >= num_blocks * page_size: skipped, recorded as
 * NVKV_DEVERR_SLOT_RANGE).  Bit-exact with the formula above.
 *
 * nvkv_paged_attention_fp8: nvkv_paged_attention over an fp8 pool (paged
 * only: block_tables required; page_size a multiple of 128; caches, scale
 * arrays, q, out and workspace 16-byte aligned).  q/out are bf16/f16 as
 * `dtype`.  Decode rows read the codes directly (half the bytes);
 * prompt rows (q_len > 1) are dequantised into the workspace first, so the
 * caller passes prompt_kv_tokens >= the sum of k_len over the batch's
 * q_len > 1 sequences (0 when max_seqlen_q <= 1); a prompt that does not fit
 * is skipped and reported as NVKV_DEVERR_SEQLEN.  The workspace holds
 * nvkv_paged_attention_fp8_workspace_size() bytes.  Outputs are the attention
 * of q over the dequantised keys and values: decode rows take S = (q . codes)
 * x k_scale and P x v_scale in f32 (q enters the products as e4m3 pieces
 * that hold it exactly down to 2^-10 of the group's largest |q|), prompt
 * rows attend over values rounded to the dtype.
 * ---------------------------------------------------------------------- */
int nvkv_store_kvcache_fp8(const void* key, const void* value, void* k_cache, void* v_cache,
                           float* k_scale, float* v_scale, const int64_t* slot_mapping,
                           int64_t num_tokens, int num_kv_heads, int head_dim,
                           int64_t key_stride, int64_t value_stride, int64_t num_blocks,
                           int page_size, int dtype, nvkv_stream_t stream);

int nvkv_paged_attention_fp8_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads,
                                            int head_dim, int max_seqlen_q, int max_seqlen_k,
                                            int64_t prompt_kv_tokens, size_t* bytes);

int nvkv_paged_attention_fp8(const void* q, int64_t q_stride, int64_t num_q_tokens,
                             const void* k_cache, const void* v_cache, const float* k_scale,
                             const float* v_scale, int64_t num_blocks, void* out,
                             const uint32_t* cu_seqlens_q, const uint32_t* cu_seqlens_k,
                             const uint32_t* block_tables, int64_t block_table_stride,
                             int num_seqs, int max_seqlen_q, int max_seqlen_k, int num_q_heads,
                             int num_kv_heads, int head_dim, int page_size, float softmax_scale,
                             int causal, int64_t prompt_kv_tokens, void* workspace,
                             size_t workspace_bytes, int dtype, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * nvkv_paged_attention without a workspace argument, for callers that cannot
 * allocate device memory on the call path (an engine that has handed nearly
 * all free GPU memory to its KV pool, code inside a stream capture that may
 * not allocate, a binding with no allocator at hand).  No counterpart in the
 * reference: its flash-attn call allocates through candle.
 * Same inputs, outputs and validation as nvkv_paged_attention.  The
 * workspace (split-KV scratch and prefill plan) is a file-scope device array of NVKV_NOALLOC_SCRATCH_BYTES held by
 * every GPU that loads the library until exit; batches whose plan needs more
 * are rejected with NVKV_ERR_WORKSPACE.  All calls share that array (it keeps
 * the last call's contents; nothing needs to start zeroed), so calls that
 * overlap on the GPU race: serialise them.  The first call on a device looks
 * the array's address up once, which (with CUDA's lazy module loading) is
 * also when the array takes its device memory: make that call before any
 * stream capture and before sizing the KV pool from free memory
 * (nvkv_kv_pool_probe); a call with num_seqs == 0 does only this set-up.  The
 * address is kept until exit, so a cudaDeviceReset after the first call is
 * not supported.  Calls no cudaMalloc/cudaFree.
 * ---------------------------------------------------------------------- */
#define NVKV_NOALLOC_SCRATCH_BYTES (4u << 20)

int nvkv_paged_attention_noalloc(const void* q, int64_t q_stride, int64_t num_q_tokens,
                                 const void* k_cache, const void* v_cache, int64_t num_blocks,
                                 int64_t kv_stride, void* out, const uint32_t* cu_seqlens_q,
                                 const uint32_t* cu_seqlens_k, const uint32_t* block_tables,
                                 int64_t block_table_stride, int num_seqs, int max_seqlen_q,
                                 int max_seqlen_k, int num_q_heads, int num_kv_heads,
                                 int head_dim, int page_size, float softmax_scale, int causal,
                                 int dtype, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused epilogues around the path (one launch each instead of candle's op
 * chains), at the reference's rounding points.
 *
 * nvkv_rms_norm replaces nanovllm_rs/src/layers/layernorm.rs:18-25
 * (RMSNorm::forward, residual == NULL) and :27-42 (residual_forward):
 *   s = x (+ residual) in f32; residual <- dtype(s) when given (in place);
 *   out = dtype(dtype(s * 1/sqrt(mean(s^2) + eps)) * weight)
 * x/residual/out: [num_tokens, hidden] rows with the given strides
 * (elements); weight [hidden].  hidden % 8 == 0, hidden <= 8192, rows 16-byte
 * aligned.
 *
 * nvkv_silu_and_mul replaces layers/activation.rs:5-17 (SiluAndMul):
 *   out[t, i] = dtype(dtype(silu(g)) * u), g = gate_up[t, i],
 *   u = gate_up[t, inter + i]; gate_up [num_tokens, 2*inter], out
 *   [num_tokens, inter].  inter % 8 == 0.
 * ---------------------------------------------------------------------- */
int nvkv_rms_norm(const void* x, int64_t x_stride, void* residual, int64_t residual_stride,
                  const void* weight, float eps, void* out, int64_t out_stride,
                  int64_t num_tokens, int hidden, int dtype, nvkv_stream_t stream);

int nvkv_silu_and_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                      int64_t num_tokens, int inter, int dtype, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * On-device sampling.  Replaces Sampler::forward
 * (nanovllm_rs/src/layers/sampler.rs:7-21: softmax(logits / T) / E,
 * E = max(-log U, 1e-10), argmax) by its Gumbel-max equivalent
 *   token = argmax_v  logit[v] / T - log(max(-log u_v, 1e-10))
 * which needs no softmax pass: the log-sum-exp the softmax subtracts is the
 * same for every v of a row.  u_v comes from Philox4x32-10 keyed by `seed`,
 * counter (global index / 4, row, step low 32 bits, step high 32 bits),
 * u = ((bits >> 9) + 1/2) 2^-23, so the noise of an element depends only on
 * (seed, step, row, global vocab index): a vocab-parallel shard
 * (vocab_offset = the global index of its column 0) gives the same
 * candidates as the whole vocabulary, and the largest value over the shards
 * (ties to the lowest index) is the whole row's sample.  Temperatures <= 0
 * give the plain arg-max (greedy).  The counter's step is `step` plus, when
 * step_device is not NULL, the int64 it points to (device memory, read by
 * the kernel): a CUDA graph that replays the call sets that word between
 * replays.
 * logits: [num_rows, row_stride] of dtype NVKV_DTYPE_BF16 / F16 / F32 (the
 * first `vocab` columns are read); temperatures [num_rows] f32; out_value
 * [num_rows] f32 (the winning score), out_index [num_rows] i64 (its global
 * vocab index).  All device memory.
 * ---------------------------------------------------------------------- */
int nvkv_sample(const void* logits, int64_t num_rows, int64_t vocab, int64_t row_stride,
                int64_t vocab_offset, const float* temperatures, uint64_t seed, uint64_t step,
                const int64_t* step_device, float* out_value, int64_t* out_index, int dtype,
                nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Device-side metadata of a pure decode step.  Replaces the decode case of
 * ModelRunner::prepare_model_input (engine/model_runner.rs:69-160) after
 * Sequence::append (engine/sequence.rs), and the H2D upload of its tensors
 * (model_runner.rs:134-146), so consecutive decode steps need no host round
 * trip.  For each of num_seqs sequences (every one decoding one token):
 *   seq_lens[b] += 1                      (last step's token is appended)
 *   positions[b] = seq_lens[b] - 1
 *   slot_mapping[b] = page * page_size + positions[b] % page_size,
 *     page = block_tables[b * block_table_stride + positions[b] / page_size]
 *     (-1 and NVKV_DEVERR_BLOCK_RANGE when that entry is past the table or
 *     page >= num_blocks: the block manager must append the page first)
 *   cu_seqlens_q[b] = b;  cu_seqlens_k = exclusive-then-total prefix sum of
 *     seq_lens ([num_seqs + 1]); seq_lens doubles as context_lens.
 * All buffers are device memory; integer arithmetic, bit-exact with the host.
 * max_seqlen_k for the attention call stays a host value: pass an upper bound
 * (e.g. the current maximum plus the number of steps a graph replays).
 * ---------------------------------------------------------------------- */
int nvkv_decode_advance(int num_seqs, int page_size, int64_t* seq_lens,
                        const uint32_t* block_tables, int64_t block_table_stride,
                        int64_t num_blocks, int64_t* positions, int64_t* slot_mapping,
                        uint32_t* cu_seqlens_q, uint32_t* cu_seqlens_k, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel epilogue: all-reduce of the row-parallel partial sums,
 * residual add and RMSNorm in ONE kernel over NVLink peer memory.
 *
 * Replaces, at each all-reduce of the decoder, the NCCL call of
 * RowParallelLinear::forward (layers/linear.rs:200-208) and of
 * VocabParallelEmbedding::forward (layers/embed_head.rs:58), made through
 * AllReduce (layers/dist_util.rs:29-84), together with the
 * RMSNorm::forward / residual_forward (layers/layernorm.rs:18-42) that
 * follows every one of them in Qwen3 (models/qwen3.rs:232-238, 295).
 *
 * One process per GPU.  Every rank creates a communicator (one device
 * allocation holding an input buffer, a gather buffer and barrier flags),
 * passes its NVKV_COMM_HANDLE_BYTES handle to every other rank over any
 * out-of-band channel (an all-gather on the process group), and opens the
 * peers' allocations (cudaIpcOpenMemHandle).  The producer of the partial
 * sums (the o_proj / down_proj GEMM, the masked embedding lookup) writes
 * them into the buffer nvkv_comm_input returns, [num_tokens, hidden]
 * contiguous; then every rank calls nvkv_allreduce_rms_norm with the same
 * num_tokens and hidden, in the same order:
 *   s = sum over ranks of input (f32, rank order, rounded once to dtype)
 *   NVKV_RESIDUAL_ADD:  r = dtype(s + residual), y = rms_norm(s + residual)
 *   NVKV_RESIDUAL_INIT: r = s,                   y = rms_norm(s)
 * (rounding points of nvkv_rms_norm), residual and out [num_tokens, hidden]
 * contiguous, identical on every rank.  Each rank reduces its 1/world share
 * of the tokens with peer loads and writes the result into every rank's
 * gather buffer with peer stores; flags in peer memory order the phases.
 * Barrier epochs live on the device, so calls may be captured in a CUDA
 * graph and replayed.  A wait that exceeds the communicator's timeout
 * (2 s by default) records NVKV_DEVERR_PEER_TIMEOUT and the kernel returns;
 * the communicator must then be destroyed and recreated on every rank.
 * world <= NVKV_COMM_MAX_RANKS, hidden % 8 == 0, hidden <= 8192,
 * num_tokens * hidden * 2 <= max_bytes.  Destroy only after every rank's last
 * call has completed (e.g. after a barrier).  No counterpart in the
 * reference for the fusion itself: there the all-reduce is an NCCL call.
 * ---------------------------------------------------------------------- */
#define NVKV_COMM_HANDLE_BYTES 64
#define NVKV_COMM_MAX_RANKS 8
#define NVKV_DEVERR_PEER_TIMEOUT 5    /* a peer missed a barrier of the comm */
#define NVKV_RESIDUAL_ADD 0
#define NVKV_RESIDUAL_INIT 1

typedef struct nvkv_comm* nvkv_comm_t;

/* Allocates this rank's buffers (zeroed flags) on the current device and
 * writes its handle (NVKV_COMM_HANDLE_BYTES) to handle_out. */
int nvkv_comm_create(int rank, int world, size_t max_bytes, nvkv_comm_t* out, void* handle_out);
/* handles: world * NVKV_COMM_HANDLE_BYTES, in rank order (this rank's own
 * entry is ignored).  Call once, before the first all-reduce. */
int nvkv_comm_open_peers(nvkv_comm_t comm, const void* handles);
/* Device address of this rank's input buffer (max_bytes). */
int nvkv_comm_input(nvkv_comm_t comm, void** ptr);
/* Barrier wait limit in nanoseconds (> 0). */
int nvkv_comm_set_timeout(nvkv_comm_t comm, int64_t timeout_ns);
int nvkv_comm_destroy(nvkv_comm_t comm);
int nvkv_allreduce_rms_norm(nvkv_comm_t comm, int64_t num_tokens, int hidden, void* residual,
                            int residual_mode, const void* weight, float eps, void* out,
                            int dtype, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * Host-side mirror of the reference's operator surface, for callers that
 * drive the path the way nanovllm_rs's Attention does: a per-thread Context
 * (utils/context.rs:4-54) published once per step, and an Attention object
 * holding its layer's KV cache (layers/attention.rs:7-21).
 * ---------------------------------------------------------------------- */

/* set_context (utils/context.rs:28-50).  All pointers are device memory and
 * must stay valid until nvkv_context_reset().  block_tables may be NULL
 * (pure prefill, model_runner.rs:127-131); slot_mapping may be NULL when no
 * cache is attached (warm-up).  context_lens is accepted and, like the
 * reference, never read by attention.  Thread-local. */
int nvkv_context_set(const uint32_t* cu_seqlens_q, const uint32_t* cu_seqlens_k, int num_seqs,
                     int max_seqlen_q, int max_seqlen_k, const int64_t* slot_mapping,
                     int64_t num_slot_entries, const int64_t* context_lens,
                     const uint32_t* block_tables, int64_t block_table_stride);
/* reset_context (utils/context.rs:52-54). */
int nvkv_context_reset(void);

typedef struct nvkv_attention* nvkv_attention_t;

/* Attention::new(scale) (layers/attention.rs:14-16). */
int nvkv_attention_create(float scale, nvkv_attention_t* out);
int nvkv_attention_destroy(nvkv_attention_t attn);
/* Attention::set_kv_cache (layers/attention.rs:18-21): caches are
 * [num_blocks, page_size, num_kv_heads, head_dim] in dtype. */
int nvkv_attention_set_kv_cache(nvkv_attention_t attn, void* k_cache, void* v_cache,
                                int64_t num_blocks, int page_size, int num_kv_heads,
                                int head_dim, int dtype);
/* Attention::forward (layers/attention.rs:24-76): stores k/v through the
 * context's slot_mapping when a cache is attached, then attends through the
 * context's block_tables (or on k/v directly when there are none).
 * q: [T, Hq, D] (token stride q_stride), k/v: [T, Hkv, D] (token strides
 * k_stride/v_stride; without a cache both strides must be equal), out:
 * [T, Hq, D] contiguous.  Scratch for split-KV is owned by the attention
 * object and grown on demand (cudaMalloc). */
int nvkv_attention_forward(nvkv_attention_t attn, const void* q, int64_t q_stride,
                           const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                           int64_t num_tokens, int num_q_heads, int num_kv_heads, void* out,
                           int dtype, nvkv_stream_t stream);

/* ------------------------------------------------------------------------
 * KV-pool block manager with prefix caching: BlockManager
 * (engine/block_manager.rs:35-287), host-only.  It hands out the page ids
 * that block_tables and slot_mapping are built from, with the reference's
 * choices (same ids, same order, same hash chain), so prefix-cache hits
 * share pages exactly as the reference's engine would.  Full blocks are
 * keyed by xxh64 (seed 0) over the previous block's hash (omitted when -1)
 * and the block's token ids, each a little-endian i64 (compute_hash,
 * :53-64; xxhash-rust 0.8.16).  Where the reference asserts (a non-empty
 * block table on allocate or get_token_layout, a hashed block under
 * may_append, a ref count below zero) or would run out of free blocks, the
 * call returns NVKV_ERR_INVALID_ARG and changes nothing.  One caller at a
 * time per manager.
 * ---------------------------------------------------------------------- */
typedef struct nvkv_block_manager* nvkv_block_manager_t;

/* The block-manager view of a Sequence (engine/sequence.rs:20-60).  The
 * caller owns both arrays; the calls update the counters and the table. */
typedef struct nvkv_block_seq {
  const uint32_t* token_ids;    /* all tokens so far (prompt + completion)  */
  int64_t num_tokens;
  int64_t num_cached_tokens;    /* Sequence::num_cached_tokens (in/out)     */
  int64_t num_new_tokens;       /* Sequence::num_new_tokens (in; the
                                   scheduler sets it; deallocate zeroes it) */
  uint32_t* block_table;        /* Sequence::block_table (in/out)           */
  int64_t block_table_len;      /* entries in use (in/out)                  */
  int64_t block_table_capacity; /* entries block_table can hold             */
} nvkv_block_seq;

/* BlockManager::compute_hash(token_ids, prefix) (:53-64); prefix -1 = none. */
int nvkv_block_hash(const int64_t* token_ids, int64_t num_tokens, int64_t prefix,
                    int64_t* hash_out);
/* BlockManager::new(num_blocks, block_size) (:44-52): all blocks free, in id order. */
int nvkv_block_manager_create(int64_t num_blocks, int64_t block_size,
                              nvkv_block_manager_t* out);
int nvkv_block_manager_destroy(nvkv_block_manager_t bm);
/* free_block_ids.len() */
int nvkv_block_manager_num_free(nvkv_block_manager_t bm, int64_t* out);
/* can_allocate(num_tokens) (:93-96) */
int nvkv_block_manager_can_allocate(nvkv_block_manager_t bm, int64_t num_tokens, int* out);
/* get_token_layout(seq) (:99-134): (tokens cached in used blocks, cached in
 * free blocks, new) for a waiting sequence. */
int nvkv_block_manager_get_token_layout(nvkv_block_manager_t bm, const nvkv_block_seq* seq,
                                        int64_t* in_used, int64_t* in_free, int64_t* fresh);
/* allocate(seq) (:136-190): prefix-cache hits, then fresh blocks for
 * num_new_tokens; advances num_cached_tokens by the hits. */
int nvkv_block_manager_allocate(nvkv_block_manager_t bm, nvkv_block_seq* seq);
/* deallocate(seq) (:193-204) */
int nvkv_block_manager_deallocate(nvkv_block_manager_t bm, nvkv_block_seq* seq);
/* can_append(seq, num_new_tokens) (:207-220) */
int nvkv_block_manager_can_append(nvkv_block_manager_t bm, const nvkv_block_seq* seq,
                                  int64_t num_new_tokens, int* out);
/* may_append(seq) (:222-284): blocks (and hashes of blocks that fill up)
 * for the num_new_tokens after num_cached_tokens of a running sequence. */
int nvkv_block_manager_may_append(nvkv_block_manager_t bm, nvkv_block_seq* seq);
/* The scheduler's running-queue pass (scheduler.rs:103-140) in one call: in
 * order, can_append(seqs[i], num_new_tokens[i]) then (if it fits) set
 * num_new_tokens and may_append.  Stops at the first sequence that does not
 * fit, with *done = its index, so the caller preempts from the back as the
 * reference does and calls again from there (*done = n: all fit). */
int nvkv_block_manager_append_batch(nvkv_block_manager_t bm, nvkv_block_seq* seqs, int64_t n,
                                    const int64_t* num_new_tokens, int64_t* done);
/* Introspection (no reference counterpart): one block's ref count, hash,
 * stored token count and used flag; the free list front to back (*count is
 * its full length, ids gets the first `capacity`); the hash map lookup. */
int nvkv_block_manager_block_info(nvkv_block_manager_t bm, int64_t block_id,
                                  int64_t* ref_count, int64_t* hash, int64_t* num_token_ids,
                                  int* used);
int nvkv_block_manager_free_ids(nvkv_block_manager_t bm, uint32_t* ids, int64_t capacity,
                                int64_t* count);
int nvkv_block_manager_lookup(nvkv_block_manager_t bm, int64_t hash, int64_t* block_id);

/* ------------------------------------------------------------------------
 * Host-side step metadata: ModelRunner::prepare_model_input and
 * prepare_block_tables (engine/model_runner.rs:53-160) for any step, from
 * the block manager's sequence views, into caller-owned (e.g. pinned host)
 * buffers.  For each sequence: input ids and positions of its
 * num_new_tokens after num_cached_tokens, cu_seqlens_q/k (+= num_new /
 * num_context tokens), context_lens, slot_mapping for the blocks from
 * num_cached_tokens / block_size on, seq_need_compute_logits (indices of
 * sequences whose context covers all their tokens and that have blocks);
 * block_tables [num_seqs, width] padded with 0 only when sum(k) > sum(q).
 * The reference's warm-up rule holds: a sequence without blocks gets no
 * slots.  *sizes is always filled; with every output pointer NULL the call
 * is a size query and returns NVKV_OK, so a caller sizes its buffers with
 * one call and fills them with a second.  Outputs:
 * input_ids/positions [num_tokens], cu_seqlens_q/k [num_seqs + 1],
 * context_lens [num_seqs], need_logits [num_need_logits], slot_mapping
 * [num_slots], block_tables [num_seqs * block_table_width].  Bit-exact.
 * ---------------------------------------------------------------------- */
typedef struct nvkv_step_sizes {
  int64_t num_tokens;         /* input_ids / positions entries           */
  int64_t num_slots;          /* slot_mapping entries                    */
  int64_t num_need_logits;    /* seq_need_compute_logits entries         */
  int64_t block_table_width;  /* max block-table length                  */
  int64_t max_seqlen_q;
  int64_t max_seqlen_k;
  int has_block_tables;       /* 1 when sum(context) > sum(new tokens)   */
} nvkv_step_sizes;

int nvkv_prepare_step(const nvkv_block_seq* seqs, int64_t num_seqs, int64_t block_size,
                      int64_t* input_ids, int64_t* positions, uint32_t* cu_seqlens_q,
                      uint32_t* cu_seqlens_k, int64_t* slot_mapping, int64_t* context_lens,
                      int64_t* need_logits, uint32_t* block_tables, int64_t capacity_tokens,
                      int64_t capacity_slots, int64_t capacity_table, nvkv_step_sizes* sizes);

/* ------------------------------------------------------------------------
 * KV-pool sizing: ModelRunner::probe_num_kvcache_blocks
 * (engine/model_runner.rs:264-284).  num_blocks = max((i64)(total *
 * utilization) - (total - free), 0) / (2 * num_layers * block_size *
 * num_kv_heads * head_dim * dtype_bytes), num_kv_heads per rank; 0 blocks
 * is an error (the reference asserts).  nvkv_kv_pool_probe reads free and
 * total from cudaMemGetInfo on the current device.  Under tensor
 * parallelism the caller takes the minimum over ranks, as the reference
 * requires before allocating.  The pool itself is 2 x num_layers tensors of
 * [num_blocks, block_size, num_kv_heads, head_dim] (model_runner.rs:286-303).
 * ---------------------------------------------------------------------- */
int nvkv_kv_pool_blocks(int64_t free_bytes, int64_t total_bytes, double gpu_memory_utilization,
                        int num_layers, int block_size, int num_kv_heads, int head_dim,
                        int dtype_bytes, int64_t* num_blocks);
int nvkv_kv_pool_probe(double gpu_memory_utilization, int num_layers, int block_size,
                       int num_kv_heads, int head_dim, int dtype_bytes, int64_t* num_blocks);

#ifdef __cplusplus
}
#endif

#endif /* NVKV_H_ */
