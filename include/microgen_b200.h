/*
 * libmicrogen_b200 — C ABI of the B200 (sm_100a) decode-step hot path for MicroGen.
 *
 * Plain pointers and sizes only. Every device pointer is a CUDA device address of
 * the current device; `stream` is a cudaStream_t (NULL = legacy default stream).
 * Every entry point returns an int status (MG_OK = 0) and never aborts or traps;
 * launches are asynchronous on `stream`. Device-side failures (a bounded wait that
 * gave up, an index out of range) are recorded in a device error word that
 * mg_device_error() reads.
 *
 * Reference interfaces replaced (paths inside the MicroGen project):
 *   microgen/backends/quantized.py:30-39   quantize_linear_layer_per_channel -> mg_quantize_rows_i8
 *   microgen/backends/quantized.py:24-27   QuantizedLinear.forward           -> mg_i8_linear
 *   microgen/backends/parallel.py:34-37    ColumnParallelLinear.forward      -> mg_i8_linear on the rank's shard
 *   microgen/backends/parallel.py:65-81    RowParallelLinear.forward (+sum)  -> mg_i8_linear_packed_rowpar +
 *                                                                            mg_rowpar_reduce_norm
 *   microgen/runtime/kv_cache.py:76-127    KVCacheState.update (torch.cat)   -> mg_rope_kv_append (paged slot write)
 *   microgen/runtime/kv_cache.py:30-40     INT8 KV (quantize_kv)             -> mg_rope_kv_append_kv8 +
 *                                                                            mg_paged_decode_attn_kv8
 *   transformers sdpa_attention_forward    decode SDPA over the cache        -> mg_paged_decode_attn
 *   microgen/backends/pytorch.py:153-155   greedy torch.argmax               -> mg_argmax_rows
 */
#ifndef MICROGEN_B200_H
#define MICROGEN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MG_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------------------------ */
#define MG_OK 0
#define MG_ERR_INVALID_ARG 1 /* a size, pointer or alignment the kernels do not accept */
#define MG_ERR_UNSUPPORTED 2 /* a shape outside what the kernels were built for */
#define MG_ERR_CUDA 3        /* a CUDA runtime call failed (mg_last_cuda_error has the code) */
#define MG_ERR_TIMEOUT 4     /* a bounded device wait gave up (peer flag, mbarrier) */
#define MG_ERR_DEVICE 5      /* a device-side check failed (index out of range) */

/* ---- linear epilogues (applied to acc*scale[n] + bias[n]) --------------------------------- */
#define MG_EPI_STORE_BF16 0  /* y[m*ldy+n] = bf16(v) */
#define MG_EPI_STORE_F32 1   /* y[m*ldy+n] = v (fp32) */
#define MG_EPI_ADD_F32 2     /* y[m*ldy+n] += v (fp32 residual stream) */
#define MG_EPI_SWIGLU_BF16 3 /* rows interleaved in 64-row gate/up groups; y[m*ldy+f] = bf16(silu(g)*u) */
#define MG_EPI_GELU_BF16 4   /* y[m*ldy+n] = bf16(gelu_tanh(v)) (GPT-2 "gelu_new") */

int mg_abi_version(void);
const char* mg_status_string(int status);
/* Last cudaError_t recorded by a failing entry point of this thread (0 if none). */
int mg_last_cuda_error(void);
/* Synchronise `stream`, then read (and when `clear` != 0 reset) the device error word.
 * *code = MG_OK or the first recorded MG_ERR_*; *info = where it was recorded. */
int mg_device_error(void* stream, int clear, int* code, int* info);

/* ---- INT8 per-output-channel quantization (bit-exact with quantized.py:30-39) -------------- */
/* w fp32 [n,k] row-major -> q int8 [n,k], scales fp32 [n]:
 *   s = max(max_k |w| / 127, 1e-8);  q = clamp(rint_half_even(w / s), -128, 127) */
int mg_quantize_rows_i8(const float* w, int64_t n, int64_t k, int8_t* q, float* scales, void* stream);

/* ---- INT8 weight-only linear (quantized.py:24-27; parallel.py shards) ---------------------- */
/* y = epilogue( x[m,k] (bf16, row stride ldx) · (q[n,k]·scales[n])ᵀ + bias[n] ), fp32 accumulate.
 * bias is fp32 [n] or NULL. k % 16 == 0, ldx % 8 == 0, 16-byte aligned x and q.
 * mg_i8_linear runs the tcgen05 tensor-core kernel on row-major codes for every m; MG_EPI_SWIGLU
 * needs n % 128 == 0 (whole 64-row gate/up pairs), otherwise the call returns MG_ERR_INVALID_ARG. */
int mg_i8_linear(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                 const float* bias, int64_t n, void* y, int64_t ldy, int epilogue, void* stream);
/* Same contract, CUDA-core kernel (one warp per output row, 128-bit weight loads). */
int mg_i8_linear_simt(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                      const float* bias, int64_t n, void* y, int64_t ldy, int epilogue, void* stream);
/* Same contract, tcgen05 kernel with an explicit split-K cluster size (1..8; 0 = automatic). */
int mg_i8_linear_tc(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* q, const float* scales,
                    const float* bias, int64_t n, void* y, int64_t ldy, int epilogue, int split_k, void* stream);

/* Tile-packed codes: the weight stored as contiguous 16 KB blocks, one per 128-row x 128-column
 * tile, tiles in (row-tile, k-block) order, zero-padded to multiples of 128:
 *   packed[((t*KB + kb)*128 + r)*128 + c] = q[(t*128 + r)*k + kb*128 + c],  KB = ceil(k/128).
 * Every weight load of the linear is then one sequential 16 KB burst. Pack once at load time. */
int64_t mg_i8_packed_bytes(int64_t n, int64_t k);
int mg_i8_pack_weights(const int8_t* q, int64_t n, int64_t k, int8_t* packed, void* stream);
/* mg_i8_linear_tc on tile-packed codes (same contract otherwise; split_k 0 = automatic). */
int mg_i8_linear_packed(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed, const float* scales,
                        const float* bias, int64_t n, void* y, int64_t ldy, int epilogue, int split_k, void* stream);

/* Stream-K form of mg_i8_linear_packed (quantized.py:24-27; the shards of parallel.py:34-37), used by the
 * decode engine for m <= 128 tokens: one wave of CTAs, each streaming an equal contiguous run of the
 * packed weight's (128-row tile, 128-column block) units; tiles shared by several CTAs are finished by the
 * CTA holding their first block, which adds the others' fp32 partials in CTA order (bit-reproducible).
 * workspace: device memory of at least mg_i8_linear_sk_workspace_bytes(m) bytes, 256-byte aligned,
 * zero-filled before its first use; every launch leaves it as it found it, so one workspace serves any
 * stream-ordered sequence of calls (calls that overlap on the GPU need separate workspaces).
 * m > 128 runs the cluster kernel of mg_i8_linear_packed (the workspace is then unused). */
int64_t mg_i8_linear_sk_workspace_bytes(int64_t m);
int mg_i8_linear_packed_sk(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                           const float* scales, const float* bias, int64_t n, void* y, int64_t ldy, int epilogue,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- fused row-parallel all-reduce over peer memory (parallel.py:65-81 + its "all-reduce") ---------
 * One communicator per rank of a tensor-parallel group (world <= 8, one process per GPU):
 *   mg_comm_create  allocates this rank's receive area (2 sets x world x slot_elems/2 64-bit words) and
 *                   writes its CUDA IPC handle (mg_comm_handle_bytes() bytes) to ipc_handle;
 *   mg_comm_open    maps every rank's area from the world handles (rank order, concatenated);
 *   mg_comm_destroy unmaps and frees.
 * mg_i8_linear_packed_rowpar runs this rank's partial of a row-parallel linear (tile-packed codes, scale
 * applied, no bias) and its epilogue stores each output tile straight into every rank's receive slot over
 * NVLink as words {two bf16 values, all-reduce epoch} (n % 128 == 0). mg_rowpar_reduce_norm waits (at most
 * MG_PEER_TIMEOUT_MS from the environment of mg_comm_create, default 1000 ms; then MG_ERR_TIMEOUT in the
 * device error word) until every word it sums carries the current epoch, sets
 * h += sum over ranks (rank order) +
 * bias, and with norm = 1 (RMSNorm, w) or 2 (LayerNorm, w, wb) writes x = bf16(norm(h)). Every rank must
 * issue the same sequence of rowpar / reduce calls. m * n <= slot_elems. */
int mg_comm_handle_bytes(void);
int mg_comm_create(int rank, int world, int64_t slot_elems, void** comm, void* ipc_handle);
int mg_comm_open(void* comm, const void* ipc_handles);
int mg_comm_destroy(void* comm);
int mg_i8_linear_packed_rowpar(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                               const float* scales, int64_t n, void* comm, int split_k, void* stream);
int mg_rowpar_reduce_norm(void* comm, float* h, const float* bias, int m, int n, int norm, const float* w,
                          const float* wb, float eps, void* x, void* stream);
/* Greedy argmax over a vocab-parallel lm_head (pytorch.py:153-155 torch.argmax over logits whose columns
 * are split across the ranks in rank order, each rank holding lm_head rows [offset, offset + n_local) —
 * the reference's split rule, n // world with the remainder on the last rank). logits: this rank's fp32
 * [m, n_local] shard (row stride ld). Finds each row's first maximal local column, exchanges {value,
 * global index} with every rank through the communicator's receive areas (two epoch-tagged words per row,
 * the same epoch sequence as the row-parallel pushes, so every rank must make this call at the same point
 * of that sequence), and writes idx[i] = the global first maximal index of row i, identical on every rank
 * (NaN counts as larger than every number, as in torch.argmax: a row with a NaN gives its first NaN).
 * m <= 1024 and 2 * m <= slot words. A peer that never publishes makes the wait give up after the
 * communicator's limit (MG_ERR_TIMEOUT in the device error word). */
int mg_vocab_argmax(void* comm, const float* logits, int m, int64_t n_local, int64_t ld, int64_t offset,
                    int32_t* idx, void* stream);
/* mg_i8_linear_packed_rowpar on the stream-K kernel (workspace as for mg_i8_linear_packed_sk). */
int mg_i8_linear_packed_rowpar_sk(const void* x, int64_t m, int64_t k, int64_t ldx, const int8_t* packed,
                                  const float* scales, int64_t n, void* comm, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ---- persistent decode layer: every linear, norm and the RoPE/KV append between two attentions -----
 * One launch replaces, for one layer boundary of a decode step (M <= 32 tokens):
 *   quantized.py:24-27 QuantizedLinear.forward of o_proj, gate/up, down_proj, q/k/v (tile-packed codes),
 *   parallel.py:40-81 RowParallelLinear + its all-reduce for o_proj and down_proj (comm != NULL),
 *   the HF post-attention norm, SwiGLU (modeling_llama.py:182-183) or GELU MLP, the next input norm, and
 *   kv_cache.py:76-127 KVCacheState.update with RoPE (one paged slot write per token).
 * Phases (flags): MG_BLK_O      h += attn · Woᵀ (+ bias)                       [attn bf16 m x hq*d]
 *                 MG_BLK_MLP    x2 = norm2(h); act = mlp(x2 · Wguᵀ); h += act · Wdᵀ (+ bias)
 *                 MG_BLK_N1     x1 = norm1(h)  (the next layer's input norm, or the final norm)
 *                 MG_BLK_QKV    q_out, K/V slots = rope(x1 · Wqkvᵀ + b)
 * Enabled phases run in that order; a phase whose producer phase is not enabled reads its input as it
 * was before the launch. norm: MG_NORM_RMS (w) or MG_NORM_LAYER (w, b). mlp: MG_EPI_SWIGLU_BF16 (gate/up
 * rows interleaved in 64-row groups) or MG_EPI_GELU_BF16. o.n = down.n = hidden and gate_up.n are
 * multiples of 128; qkv.n = (hq + 2*hkv) * head_dim (any multiple of 16: the packed codes are zero-padded
 * to whole tiles); every k a multiple of 16; head_dim in {32, 64, 128}; cos_sin NULL = no RoPE (GPT-2).
 * comm (world > 1, from mg_comm_create/open): o and down are this rank's row-parallel shards; their
 * tiles are pushed to every rank and the norm sums them in rank order (bias once), as
 * mg_i8_linear_packed_rowpar + mg_rowpar_reduce_norm do; NULL = world 1.
 * workspace: mg_decode_block_workspace_bytes() bytes, 256-byte aligned, zero-filled before its first use.
 * Its first 64 KB are control words (tile tickets, flags, phase counters) that every launch leaves at zero;
 * the split partials follow. So one workspace serves any stream-ordered sequence of launches whose plans
 * fit in it, the different plans of a model's layer boundaries included. One CTA per SM; the launch assumes the whole GPU (a CTA that cannot
 * become resident makes the others' bounded waits give up with MG_ERR_TIMEOUT). */
#define MG_NORM_RMS 1
#define MG_NORM_LAYER 2
#define MG_BLK_O 1
#define MG_BLK_MLP 2
#define MG_BLK_N1 4
#define MG_BLK_QKV 8
typedef struct mg_block_linear {
  const int8_t* packed; /* tile-packed codes of [n, k] (mg_i8_pack_weights) */
  const float* scales;  /* [n] */
  const float* bias;    /* [n] or NULL */
  int64_t n, k;
} mg_block_linear;
typedef struct mg_block_args {
  int m, flags, hidden, hq, hkv, head_dim, norm, mlp;
  float eps;
  int max_pos;
  mg_block_linear o, gate_up, down, qkv;
  float* h;                         /* fp32 [m, hidden] residual stream, updated in place */
  const void* attn;                 /* bf16 [m, hq*head_dim]: the o_proj input */
  const float* n2_w; const float* n2_b;
  void* x2;                         /* bf16 [m, hidden]: norm2 output */
  void* act;                        /* bf16 [m, down.k]: MLP activation */
  const float* n1_w; const float* n1_b;
  void* x1;                         /* bf16 [m, hidden]: norm1 output (QKV input, or lm_head input) */
  const float* cos_sin;             /* fp32 [max_pos, head_dim] (cos | sin) or NULL */
  const int32_t* positions;         /* [m] */
  const int32_t* slots;             /* [m] paged slot of the new token */
  float* q_out;                     /* fp32 [m, hq, head_dim] */
  void* k_pool; void* v_pool;       /* bf16 [num_blocks, hkv, 16, head_dim] of the QKV phase's layer */
  int64_t num_blocks;
} mg_block_args;
int mg_decode_block_workspace_bytes(const mg_block_args* args, size_t* bytes);
int mg_decode_block(const mg_block_args* args, void* comm, void* workspace, size_t workspace_bytes, void* stream);
/* Diagnosis of the first bounded wait of mg_decode_block that gave up on the current device (MG_ERR_TIMEOUT
 * in the device error word): out[0] = site (0 = none), [1] CTA, [2] thread, [3..4] site-specific words,
 * [8..15] the launch's first eight control words; out[32 + 4*c + r]: the
 * progress of CTA c < 256 in role r (0 producer, 1 converters, 2 MMA, 3 epilogue) when that wait gave
 * up. out holds 32 + 1024 words. Synchronous; clear != 0 resets the first 32. */
int mg_decode_block_diag(uint32_t* out32, int clear);
/* Timeline of the latest mg_decode_block launch on the current device: out[16*c + k] = globaltimer (ns)
 * of CTA c (< ctas <= 256) at point k — 0 entry, 1 dependency released, 2..5 first activation tile of
 * o_proj / gate-up / down / QKV requested, 6 last MMA issued, 7 epilogue start, 8 o_proj drained,
 * 9 norm2 done, 10 gate/up drained, 11 down drained, 12 norm1 done, 13 QKV drained, 14 last weight
 * tile converted, 15 exit. Points a launch does not reach keep older values. Synchronous. */
int mg_decode_block_trace(uint64_t* out, int ctas);

/* ---- paged KV: RoPE + append (kv_cache.py:76-127, as one slot write per token) ------------ */
/* qkv fp32 [b, (hq+2*hkv)*d] (row stride ld_qkv): q heads, then k heads, then v heads.
 * rope: cos_sin fp32 [max_pos, d] (cos of the d/2 frequencies, then sin), NULL = no rotation.
 * Writes q_out fp32 [b, hq, d] (rotated) and K/V (rotated K) into the pools
 * bf16 [num_blocks, hkv, 16, d] at slot_mapping[i] = block_id*16 + offset. */
int mg_rope_kv_append(const float* qkv, int64_t ld_qkv, const int32_t* positions, const float* cos_sin,
                      int max_pos, const int32_t* slot_mapping, int b, int hq, int hkv, int d, float* q_out,
                      void* k_pool, void* v_pool, int64_t num_blocks, void* stream);

/* ---- paged decode attention ---------------------------------------------------------------- */
/* out bf16 [b, hq*d] = softmax(q·Kᵀ·scale)·V per sequence, query head h reading kv head
 * h / (hq/hkv); K/V gathered through block_tables int32 [b, max_blocks] from pools
 * bf16 [num_blocks, hkv, 16, d]; ctx_lens int32 [b] >= 1. d in {32, 64, 128}; hq/hkv <= 16.
 * n_shared_blocks: the first n_shared_blocks entries of every table are the same blocks
 * (a shared prefix); they are read once per batch. 0 = no sharing. A table whose leading entries differ
 * from row 0's is recorded as MG_ERR_DEVICE (site 403).
 * workspace: device scratch of mg_paged_attn_workspace_bytes() bytes (may be NULL if 0). When the launch
 * splits a sequence's blocks over several CTAs, a second kernel merges the split partials (log-sum-exp). */
int mg_paged_attn_workspace_bytes(int b, int hq, int hkv, int d, int max_blocks, int n_shared_blocks,
                                  size_t* bytes);
int mg_paged_decode_attn(const float* q, const void* k_pool, const void* v_pool, int64_t num_blocks,
                         const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens, int b, int hq,
                         int hkv, int d, int n_shared_blocks, float scale, void* out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* ---- paged INT8 KV (kv_cache.py:30-40, 114-120: KVCacheState with quantize_kv) ------------------
 * Pools int8 [num_blocks, hkv, 16, d] and one fp32 scale per (block, kv head, token) vector in
 * k_scales / v_scales [num_blocks, hkv, 16] (16-byte aligned). mg_rope_kv_append_kv8: as
 * mg_rope_kv_append, then each K and V vector of d values x is stored as s = max(max|x| / 127, 1e-8),
 * code = clamp(round_half_even(x / s), -128, 127) — the reference's _quantize_tensor over head_dim.
 * mg_paged_decode_attn_kv8: as mg_paged_decode_attn over those pools, with K and V the codes times their
 * scales (the codes enter the tensor cores exactly; the scales multiply the scores and the probabilities).
 * Workspace bytes as mg_paged_attn_workspace_bytes. The step's own token is read back quantized, where the
 * reference attends to it before quantizing. */
int mg_rope_kv_append_kv8(const float* qkv, int64_t ld_qkv, const int32_t* positions, const float* cos_sin,
                          int max_pos, const int32_t* slot_mapping, int b, int hq, int hkv, int d, float* q_out,
                          int8_t* k_pool, int8_t* v_pool, float* k_scales, float* v_scales, int64_t num_blocks,
                          void* stream);
int mg_paged_decode_attn_kv8(const float* q, const int8_t* k_pool, const int8_t* v_pool, const float* k_scales,
                             const float* v_scales, int64_t num_blocks, const int32_t* block_tables, int max_blocks,
                             const int32_t* ctx_lens, int b, int hq, int hkv, int d, int n_shared_blocks,
                             float scale, void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free paged decode attention. No counterpart in the reference: it exists for callers that
 * cannot allocate device memory themselves — a host binding that only receives pointers from another
 * runtime's allocator, or a serving loop that must not take cudaMalloc's device-wide synchronisation in
 * the middle of a step. Same contract as mg_paged_decode_attn, but the split scratch is a fixed
 * library-owned device array of MG_ATTN_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps
 * until the process exits; the caller still passes q, the pools, the tables, ctx_lens and `out`.
 * Limit: returns MG_ERR_UNSUPPORTED when mg_paged_attn_workspace_bytes() for the sizes exceeds the array.
 * Allocates nothing (no cudaMalloc / cudaFree / allocating library call). The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress, once per device, with that device current);
 * make that first call before any stream capture. The address is kept for the life of the process:
 * after cudaDeviceReset (which unloads the library's device code) this entry point must not be called
 * again on that device. All calls share the array: calls whose kernels overlap on the GPU (e.g. on two
 * streams) race on it — serialise them. Nothing in it needs clearing: each call writes every slot it
 * later reads (a split whose bounded wait gave up writes an empty softmax state and records
 * MG_ERR_TIMEOUT). */
#define MG_ATTN_NOALLOC_SCRATCH_BYTES (16u << 20)
int mg_paged_decode_attn_noalloc(const float* q, const void* k_pool, const void* v_pool, int64_t num_blocks,
                                 const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens, int b,
                                 int hq, int hkv, int d, int n_shared_blocks, float scale, void* out,
                                 void* stream);

/* ---- small fused ops of the decode step ---------------------------------------------------- */
/* h fp32 [b, hidden] = wte[tokens[i]] (+ wpe[positions[i]] when wpe != NULL). */
int mg_embed(const int32_t* tokens, const int32_t* positions, const float* wte, const float* wpe, int b,
             int hidden, int64_t vocab, int max_pos, float* h, void* stream);
/* x bf16 [m, n] = w * h * rsqrt(mean(h^2) + eps)  (LlamaRMSNorm / Qwen2RMSNorm) */
int mg_rmsnorm(const float* h, const float* w, int m, int n, float eps, void* x, void* stream);
/* x bf16 [m, n] = (h - mean) * rsqrt(var + eps) * w + bias  (GPT-2 LayerNorm) */
int mg_layernorm(const float* h, const float* w, const float* bias, int m, int n, float eps, void* x,
                 void* stream);
/* out[i] = first index of the maximum of logits fp32 row i (row stride ld) — torch.argmax, NaN counting as
 * larger than every number (a row with a NaN gives its first NaN; a row of -inf gives 0). */
int mg_argmax_rows(const float* logits, int m, int64_t n, int64_t ld, int32_t* out, void* stream);
/* One greedy step forward for a graph-replayed decode loop: tokens = next; positions += 1;
 * ctx_lens += 1; slots = table[pos/16]*16 + pos%16 for the new position. */
int mg_decode_advance(int32_t* tokens, const int32_t* next_tokens, int32_t* positions, int32_t* ctx_lens,
                      int32_t* slots, const int32_t* block_tables, int max_blocks, int b, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MICROGEN_B200_H */
