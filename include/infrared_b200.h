/*
 * infrared_b200 — C ABI of the B200 paged-decode attention path.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, element
 * counts and strides (in elements, 64-bit), launches only on the given
 * stream, never synchronises and never allocates, so every call can sit
 * inside a CUDA graph capture. The caller owns every buffer, including the
 * workspace of the decode calls (size it with ir_paged_decode_workspace_size).
 *
 * Return value: IR_OK (0) or a non-zero IR_ERR_* status for a bad argument,
 * an unsupported shape or a CUDA launch error; ir_last_error() gives the
 * message of the calling thread's last failure. Errors found on the device
 * (a block id or slot outside the pool, a context longer than the block
 * table, metadata that is not block structured) never trap: the kernel
 * skips the access and ORs an IR_DEVERR_* bit into the caller's int32
 * `err_flag` word, which the host reads when it chooses (outside capture).
 *
 * Pool layout (one layer): k_pool / v_pool are [num_slots, num_kv_heads,
 * head_dim] contiguous, slot = block_id * block_size + offset — the layout of
 * PagedKVPool (infrared/cache/paged_kv_cache.py:30-46) with the layer index
 * already applied by the caller (pointer of pool.k[layer]).
 */
#ifndef INFRARED_B200_H_
#define INFRARED_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ir_stream_t; /* == cudaStream_t */

/* element types */
#define IR_DTYPE_F32 0
#define IR_DTYPE_BF16 1
#define IR_DTYPE_F16 2

/* host-side status codes */
#define IR_OK 0
#define IR_ERR_INVALID_ARG 1
#define IR_ERR_UNSUPPORTED 2
#define IR_ERR_CUDA 3
#define IR_ERR_WORKSPACE 4

/* device-side error bits ORed into *err_flag */
#define IR_DEVERR_BLOCK_ID 0x1      /* block table entry outside [0, num_blocks) */
#define IR_DEVERR_CONTEXT_LEN 0x2   /* context_len < 0 or > max_blocks * block_size */
#define IR_DEVERR_SLOT 0x4          /* slot_mapping entry outside [0, num_slots) */
#define IR_DEVERR_NOT_BLOCKED 0x8   /* gather_slots row is not block structured */
#define IR_DEVERR_MASK 0x10         /* decode mask row is not a prefix of zeros */
#define IR_DEVERR_TIMEOUT 0x20      /* a pipeline wait ran past its time limit */
#define IR_DEVERR_WRITE_SLOT 0x40   /* fused write: slot is not the tail position */

/* Library version (major*10000 + minor*100 + patch). */
int ir_version(void);

/* Message of the calling thread's last failed call ("" if none). */
const char* ir_last_error(void);

/* Number of device-side error bits, names by bit index (0-based). */
const char* ir_deverr_name(int bit);

/*
 * Scatter this step's new K/V rows into the pool:
 *   k_pool[slot_mapping[i], h, :] = k[i, h, :]   (same for v)
 * Replaces PagedKVPool.write (infrared/cache/paged_kv_cache.py:48-57).
 * k, v: [num_tokens, num_kv_heads, head_dim] with row stride k_stride /
 * v_stride (elements) between tokens and [num_kv_heads, head_dim]
 * contiguous. A negative slot skips the row (padding); a slot >= num_slots
 * is skipped and flagged IR_DEVERR_SLOT. Duplicate slots: the rows must be
 * identical (CUDA-graph pad rows repeat row 0), otherwise which row lands is
 * unspecified.
 */
int ir_cache_write(const void* k, const void* v, int64_t k_stride,
                   int64_t v_stride, void* k_pool, void* v_pool,
                   const int64_t* slot_mapping, int64_t num_tokens,
                   int num_kv_heads, int head_dim, int64_t num_slots,
                   int dtype, int32_t* err_flag, ir_stream_t stream);

/*
 * Gather pool rows by slot: out[i, h, :] = pool[slots[i], h, :].
 * Replaces PagedKVPool.gather (infrared/cache/paged_kv_cache.py:59-72) for
 * one of k or v; out is [num_rows, num_kv_heads, head_dim] contiguous. A
 * slot outside [0, num_slots) gives a zero row and sets IR_DEVERR_SLOT.
 */
int ir_cache_gather(void* out, const void* pool, const int64_t* slots,
                    int64_t num_rows, int num_kv_heads, int head_dim,
                    int64_t num_slots, int dtype, int32_t* err_flag,
                    ir_stream_t stream);

/*
 * Fixed-shape inputs of a CUDA-graph decode step, built on the device.
 * Replaces the per-element Python loops of build_decode_static_inputs
 * (infrared/engine/cuda_graph.py:105-155) with the same outputs, bit for bit:
 * for row i < bucket, sequence j = (i < batch ? i : 0) (pad rows repeat
 * row 0), with ctx = num_cached[j] + 1 and slot(p) =
 * block_tables[j, p / block_size] * block_size + p % block_size:
 *   ids[i] = last_tokens[j]; positions[i] = num_cached[j];
 *   write_slots[i] = slot(num_cached[j]);
 *   gather_slots[i, p] = p < ctx ? slot(p) : 0                  (int64 [bucket, t_max])
 *   mask[i, 0, 0, p]  = p < ctx ? 0 : finfo(mask_dtype).min      ([bucket, 1, 1, t_max])
 * block_tables is int32 [batch, >= ceil(t_max / block_size)] with row stride
 * bt_stride; the caller guarantees ctx <= t_max (the reference raises).
 */
int ir_build_decode_inputs(const int32_t* block_tables, int64_t bt_stride,
                           const int32_t* num_cached, const int64_t* last_tokens,
                           int batch, int bucket, int64_t t_max, int block_size,
                           int64_t* ids, int64_t* positions, int64_t* write_slots,
                           int64_t* gather_slots, void* mask, int mask_dtype,
                           ir_stream_t stream);

/*
 * Turn the reference seam's per-forward metadata into block form.
 * gather_slots [B, T] int64 (row stride gs_stride) and the additive decode
 * mask [B, 1, 1, T] (row stride mask_stride, dtype mask_dtype) as built by
 * PagedBatchEngine._decode_logits_eager (infrared/engine/paged_engine.py:
 * 300-315) or build_decode_static_inputs (infrared/engine/cuda_graph.py:
 * 105-155) become
 *   context_lens[b]       = number of zero mask columns of row b
 *   block_tables[b, j]    = gather_slots[b, j*block_size] / block_size
 *                           (0 for blocks past the context)
 * block_tables is [B, ceil(T/block_size)] int32 with row stride bt_stride.
 * Rows whose valid slots are not bt[p/bs]*bs + p%bs set
 * IR_DEVERR_NOT_BLOCKED; masks that are not a prefix of zeros set
 * IR_DEVERR_MASK.
 */
int ir_derive_block_metadata(const int64_t* gather_slots, int64_t gs_stride,
                             const void* mask, int64_t mask_stride,
                             int mask_dtype, int batch, int64_t t,
                             int block_size, int32_t* block_tables,
                             int64_t bt_stride, int32_t* context_lens,
                             int32_t* err_flag, ir_stream_t stream);

/* Shape of one decode call (shared by the decode entry points). */
typedef struct ir_decode_shape {
  int batch;          /* B sequences, one query token each */
  int num_heads;      /* H query heads */
  int num_kv_heads;   /* Hkv; H % Hkv == 0, group = H / Hkv (<= 16) */
  int head_dim;       /* D: 64 or 128 */
  int block_size;     /* tokens per block */
  int max_blocks;     /* columns of block_tables that may be read */
  int64_t bt_stride;  /* row stride of block_tables (elements) */
  int64_t q_stride;   /* stride between sequences in q (elements); [H, D] contiguous */
  int64_t out_stride; /* stride between sequences in out (elements) */
  int64_t num_slots;  /* rows of the pool (num_blocks * block_size) */
  float scale;        /* softmax scale, usually head_dim ** -0.5 */
  int dtype;          /* IR_DTYPE_* of q, pools and out */
  int flags;          /* IR_DECODE_DYNAMIC_TAIL | IR_DECODE_INLINE_MERGE or 0;
                         other bits are rejected */
} ir_decode_shape;

/* ir_decode_shape.flags: the workspace was zero-filled when it was first
 * used (cudaMemset once after allocating it). The TMA
 * kernel then hands out the last ~15 % of the tiles as small units that CTAs
 * claim from counters in that header as they finish their static share, which
 * evens out the SMs' random differences in streaming speed; every call leaves
 * the header zero again. Without the flag the workspace needs no
 * initialisation and every CTA streams a fixed share. The flag changes the
 * workspace size (more partial slots); results are deterministic either way
 * (they do not depend on which CTA took which unit). */
#define IR_DECODE_DYNAMIC_TAIL 1
/* ir_decode_shape.flags: the workspace was zero-filled when it was first
 * used. The TMA kernel then merges a sequence split into at most 4 pieces
 * inside the decode kernel: the warp that writes the row's last piece folds
 * the pieces (counted in the workspace header, which every call leaves zero
 * again) while the other CTAs are still streaming, instead of the separate
 * merge kernel doing it after the decode has finished (num_kv_heads * batch
 * up to 16384; larger shapes leave every row to the merge kernel). The
 * header sits at the start of the workspace in every layout, so one zeroed
 * workspace may serve calls of any shape and flags. */
#define IR_DECODE_INLINE_MERGE 2

/* Bytes of workspace the decode calls need for this shape on the current
 * device (0 on an invalid shape). The workspace holds the tile prefix and the
 * partial results of sequences split across CTAs; it must be 256-byte
 * aligned and needs no initialisation unless shape->flags asks for the
 * dynamic tail. Calls sharing a workspace must not overlap on the GPU (calls
 * on one stream never do). */
size_t ir_paged_decode_workspace_size(const ir_decode_shape* shape);

/* Kernel choice for this shape on the current device: *path = 1 (CUDA-core
 * kernel: fp32, groups of 9-16, other block sizes) or 2 (TMA + mma kernel:
 * bf16/fp16, group <= 8, block_size 8 or a multiple of 16), and the number
 * of CTAs each kv head's tiles are divided among. No reference counterpart
 * (the gate of the reference is _should_use_triton,
 * infrared/model/triton_attention.py:68-76). */
int ir_paged_decode_plan(const ir_decode_shape* shape, int* path,
                         int* ctas_per_kv_head);

/* Process-wide kernel override for testing and tuning: 0 = automatic,
 * 1 = always the CUDA-core kernel, 2 = the TMA kernel (calls whose shape is
 * not eligible then fail with IR_ERR_UNSUPPORTED), 3 = the TMA kernel with
 * one tensor copy per (kv head, 64-column half) instead of one per tile. */
int ir_set_decode_path(int path);

/* Test hook of the failure path (no reference counterpart): the next launch
 * of the TMA decode kernel makes its first CTA wait for 16 bytes that no copy
 * delivers. Its bounded waits run out after about two seconds, the kernel
 * sets IR_DEVERR_TIMEOUT and returns (that call's output is undefined); the
 * context stays usable. Nothing faults, traps or hangs. */
int ir_debug_stall_next_decode(void);

/*
 * Decode attention of one query token per sequence over its paged history:
 *   out[b, h, :] = softmax_j(q[b, h, :] . K[slot_j, h / G, :] * scale) V[slot_j, h / G, :]
 * over the context_lens[b] positions j whose slots come from block_tables.
 * Replaces the decode read of paged_attention (infrared/model/
 * triton_attention.py:81-107): _paged_attention_naive (:110-129) and
 * _paged_attention_triton (:310-359). A sequence with context_len 0 gets a
 * zero row (the l_safe convention of the reference kernel, :293-297).
 * Work is split across the GPU's SMs in equal token shares; the pieces of a
 * sequence that spans several CTAs are combined (log-sum-exp) by a merge
 * kernel launched behind the decode kernel with programmatic dependent
 * launch (two launches per call, one stream).
 */
int ir_paged_decode(void* out, const void* q, const void* k_pool,
                    const void* v_pool, const int32_t* block_tables,
                    const int32_t* context_lens, const ir_decode_shape* shape,
                    void* workspace, size_t workspace_bytes,
                    int32_t* err_flag, ir_stream_t stream);

/*
 * ir_paged_decode fused with the cache write of this step's K/V:
 * k_new / v_new [B, Hkv, D] (row stride kv_stride) are written to pool slot
 * slot_mapping[b] and used as the key/value of position context_lens[b]-1.
 * slot_mapping[b] must be the tail slot of sequence b (the engine's
 * invariant, infrared/engine/paged_engine.py:303-305); otherwise
 * IR_DEVERR_WRITE_SLOT is set. Replaces the write + read of paged_attention
 * (infrared/model/triton_attention.py:100-107) in one launch.
 */
int ir_paged_decode_write(void* out, const void* q, void* k_pool, void* v_pool,
                          const void* k_new, const void* v_new,
                          int64_t kv_stride, const int64_t* slot_mapping,
                          const int32_t* block_tables,
                          const int32_t* context_lens,
                          const ir_decode_shape* shape, void* workspace,
                          size_t workspace_bytes, int32_t* err_flag,
                          ir_stream_t stream);

/*
 * ir_paged_decode_write with rotary position embedding applied inside the
 * kernel: q and k_new are the UN-rotated projections; the kernel rotates q
 * (in registers) and the new K row (before it is stored in the pool and
 * used) as infrared's apply_rotary_pos_emb does
 * (infrared/model/layers.py:79-89: q * cos + rotate_half(q) * sin with the
 * fp32 cos/sin tables cast to the dtype, each op rounded to the dtype), so
 * the pool and the output equal rotate-then-ir_paged_decode_write exactly.
 * rope_cos / rope_sin: fp32 [batch, head_dim] rows with row stride
 * rope_stride elements (infrared's RotaryEmbedding output at the new
 * token's position, infrared/model/layers.py:121-136). q, k_new and v_new
 * may be row views of one fused QKV projection output (q_stride in shape,
 * kv_stride here). Replaces apply_rotary_pos_emb + write + read of
 * Attention.forward (infrared/model/layers.py:165-181) in one launch.
 */
int ir_paged_decode_rope_write(void* out, const void* q, void* k_pool, void* v_pool,
                               const void* k_new, const void* v_new,
                               int64_t kv_stride, const int64_t* slot_mapping,
                               const float* rope_cos, const float* rope_sin,
                               int64_t rope_stride, const int32_t* block_tables,
                               const int32_t* context_lens,
                               const ir_decode_shape* shape, void* workspace,
                               size_t workspace_bytes, int32_t* err_flag,
                               ir_stream_t stream);

/*
 * ir_paged_decode with RoPE applied to q in the kernel (fp32 cos/sin rows
 * [B, head_dim] with rope_stride, as infrared's RotaryEmbedding returns them):
 * for a step whose new K/V are already in the pool (ir_kv_proj_rope_write).
 * Replaces apply_rotary_pos_emb on q (infrared/model/layers.py:79-89, 165)
 * and the read of paged_attention (infrared/model/triton_attention.py:81-129).
 */
int ir_paged_decode_rope(void* out, const void* q, const void* k_pool, const void* v_pool,
                         const float* rope_cos, const float* rope_sin, int64_t rope_stride,
                         const int32_t* block_tables, const int32_t* context_lens,
                         const ir_decode_shape* shape, void* workspace,
                         size_t workspace_bytes, int32_t* err_flag, ir_stream_t stream);

/*
 * K/V projection of num_tokens new tokens with bias, RoPE on K and the cache
 * write in one kernel (5th-generation tensor cores): for token t,
 *   k = x[t] @ w_k^T + b_k,  v = x[t] @ w_v^T + b_v   (rounded to dtype once),
 *   k = k * cos[t] + rotate_half(k) * sin[t]          (dtype rounding per op),
 *   k_pool[slot_mapping[t]] = k,  v_pool[slot_mapping[t]] = v.
 * x [num_tokens, hidden] with row stride x_stride; w_k / w_v
 * [num_kv_heads * head_dim, hidden] row-major (nn.Linear weights); b_k / b_v
 * [num_kv_heads * head_dim] or null; rope_cos / rope_sin fp32 rows
 * [num_tokens, head_dim] with rope_stride, or null (no RoPE). bf16 / fp16,
 * head_dim 64 or 128, hidden a multiple of 64; x, the weights and the pools
 * 16-byte aligned. A slot outside the pool is skipped and flagged
 * (IR_DEVERR_SLOT). Replaces k_proj / v_proj, apply_rotary_pos_emb on k of
 * Attention.forward (infrared/model/layers.py:158-165) and PagedKVPool.write
 * (infrared/cache/paged_kv_cache.py:48-57).
 */
int ir_kv_proj_rope_write(const void* x, int64_t x_stride, int num_tokens, int hidden,
                          const void* w_k, const void* w_v, const void* b_k,
                          const void* b_v, const float* rope_cos, const float* rope_sin,
                          int64_t rope_stride, const int64_t* slot_mapping, void* k_pool,
                          void* v_pool, int64_t num_slots, int num_kv_heads, int head_dim,
                          int dtype, int32_t* err_flag, ir_stream_t stream);

/*
 * Decode attention returning the softmax-normalised fp32 output and its
 * log-sum-exp instead of the final row: o [B, H, D] fp32 contiguous,
 * lse [B, H] fp32 natural log (-inf for an empty context, o = 0). These are
 * the partials of a KV range held on one GPU; ir_lse_merge combines ranges.
 * No reference counterpart: the reference defers split-KV
 * (infrared docs/research/t4-triton-cudagraph-api.md:130).
 */
int ir_paged_decode_lse(float* o, float* lse, const void* q,
                        const void* k_pool, const void* v_pool,
                        const int32_t* block_tables,
                        const int32_t* context_lens,
                        const ir_decode_shape* shape, void* workspace,
                        size_t workspace_bytes, int32_t* err_flag,
                        ir_stream_t stream);

/* Largest workspace ir_paged_decode_noalloc can serve (bytes). */
#define IR_NOALLOC_WORKSPACE_BYTES (8u << 20)

/*
 * ir_paged_decode for callers that cannot allocate device memory. No
 * counterpart in the reference (its path allocates through PyTorch).
 *
 * Some hosts own every device byte themselves and forbid allocation calls on
 * their serving path: an engine that hands out a fixed memory budget at
 * start-up, a plugin loaded into another runtime's process, or a foreign-
 * language binding with no access to a device allocator. They cannot supply
 * the workspace ir_paged_decode asks for. This entry point takes the same
 * inputs and outputs but keeps its scratch (partial results of sequences
 * split across SMs) in an 8 MiB array that is part of the library itself
 * (IR_NOALLOC_WORKSPACE_BYTES; every GPU that loads the library holds it
 * until the process exits). It calls no cudaMalloc or cudaFree.
 *
 * - The first call on a device looks up the array's device address with
 *   that device current (this may load the library's GPU code), so make that
 *   first call before capturing a CUDA graph. The address is looked up
 *   again when the device's context has changed since (after a device
 *   reset), so make the first call after a reset outside capture too.
 * - Shapes whose scratch (ir_paged_decode_workspace_size) exceeds
 *   IR_NOALLOC_WORKSPACE_BYTES are rejected with IR_ERR_WORKSPACE.
 * - All calls on a device share the one array and it keeps whatever the
 *   last call left in it; nothing in it needs to start at zero. Calls that
 *   may run at the same time on the GPU (different streams without ordering
 *   between them) race on it and give wrong results: order them.
 */
int ir_paged_decode_noalloc(void* out, const void* q, const void* k_pool,
                            const void* v_pool, const int32_t* block_tables,
                            const int32_t* context_lens,
                            const ir_decode_shape* shape, int32_t* err_flag,
                            ir_stream_t stream);

/*
 * Combine P partials: out[b, h, :] = sum_p w_p o_parts[p, b, h, :] with
 * w_p = exp(lse_parts[p, b, h] - LSE), LSE = log sum_p exp(lse_parts[p]).
 * Part p of o_parts starts at o_parts + p * o_part_stride and is [B, H, D]
 * fp32 contiguous; part p of lse_parts starts at lse_parts + p *
 * lse_part_stride and is [B, H] (strides in elements: B*H*D and B*H for
 * stacked arrays, or the packed row of an all-gather). out is [B, H, D] of
 * `dtype` with sequence stride out_stride. Rows whose partials are all -inf
 * become zero. No reference counterpart (the reference defers split-KV,
 * infrared docs/research/t4-triton-cudagraph-api.md:130).
 */
int ir_lse_merge(void* out, int64_t out_stride, const float* o_parts,
                 int64_t o_part_stride, const float* lse_parts,
                 int64_t lse_part_stride, int num_parts, int batch,
                 int num_heads, int head_dim, int dtype, ir_stream_t stream);

/* ---------------------------------------------------------- prefill
 *
 * Paged attention of packed query rows (prefill with a cached prefix, and
 * infrared's mixed prefill + decode steps): sequence s owns query rows
 * [q_start[s], q_start[s+1]) of q [total_q, H, D], which are its LAST q_len
 * positions ctx - q_len .. ctx - 1 (ctx = context_lens[s], the history length
 * after this step's K/V were written to the pool). The row at position p
 * attends positions 0..p of its own sequence, read through block_tables[s].
 * Replaces infrared's read path for Sq > 1 (_paged_attention_naive,
 * infrared/model/triton_attention.py:110-129, with the causal mask of
 * infrared/model/inputs.py:38-61 or the packed-frame mask of :64-94, as
 * built by infrared/engine/paged_engine.py:197-221 and :461-516).
 */
typedef struct ir_prefill_shape {
  int num_seqs;     /* S: sequences in the frame */
  int total_q;      /* packed query rows */
  int num_heads;    /* H */
  int num_kv_heads; /* Hkv, divides H */
  int head_dim;     /* 64 or 128 */
  int block_size;
  int max_blocks;   /* columns of block_tables */
  int64_t bt_stride;
  int64_t q_stride;   /* elements between query rows (>= H * D) */
  int64_t out_stride; /* elements between output rows (>= H * D) */
  int64_t num_slots;  /* rows of one layer's pool */
  float scale;
  int dtype;          /* IR_DTYPE_* */
} ir_prefill_shape;

/* Kernel choice for ir_paged_prefill: 0 auto, 1 rows as decode rows (every
 * query row decoded as its own sequence; any dtype), 2 the tcgen05 tensor-core
 * kernel (bf16/fp16, power-of-two block sizes >= 8), 3 its CTA-pair form
 * (the same, head_dim 128: two SMs share 256-row query tiles through
 * cta_group::2 MMAs, each staging half of every K/V tile; only on request,
 * as it measures slower). Auto picks 2 when eligible, else 1. Process-wide;
 * a test and tuning hook. */
int ir_set_prefill_path(int path);

/* Path (1, 2 or 3) ir_paged_prefill takes for this shape. */
int ir_paged_prefill_plan(const ir_prefill_shape* shape, int* path);

/* Workspace bytes ir_paged_prefill needs (0 for the tensor-core path). */
size_t ir_paged_prefill_workspace_size(const ir_prefill_shape* shape);

/* out[t, h, :] for every packed query row t. context_lens and q_start are
 * int32 device arrays; a sequence with context_lens < q_len (or past the
 * block table) sets IR_DEVERR_CONTEXT_LEN and its rows are not valid output;
 * bad block ids read zeros and set IR_DEVERR_BLOCK_ID. */
int ir_paged_prefill(void* out, const void* q, const void* k_pool, const void* v_pool,
                     const int32_t* block_tables, const int32_t* context_lens,
                     const int32_t* q_start, const ir_prefill_shape* shape, void* workspace,
                     size_t workspace_bytes, int32_t* err_flag, ir_stream_t stream);

/*
 * The block-table form of one packed frame as infrared's engine builds it
 * for Sq > 1 (prefill with a cached prefix, paged_engine.py:197-221; the
 * mixed step, :461-516): gather_slots int64 [num_keys] (the histories of the
 * frame's sequences laid end to end) and the additive mask
 * [num_rows, num_keys] (row stride mask_stride elements; 0 = allowed) of
 * infrared/model/inputs.py:38-94. Writes block_tables [num_rows, max_blocks]
 * (row s for sequence s), context_lens [num_rows], q_start [num_rows + 1]
 * and *num_seqs (all device memory); scratch: 3 * num_rows int32. A mask
 * row that is not one contiguous range, or a sequence whose rows do not
 * advance by one position, sets IR_DEVERR_MASK; slots that are not block
 * structured set IR_DEVERR_NOT_BLOCKED.
 */
int ir_derive_varlen_metadata(const int64_t* gather_slots, int64_t num_keys, const void* mask,
                              int64_t mask_stride, int mask_dtype, int num_rows,
                              int block_size, int max_blocks, int32_t* block_tables,
                              int32_t* context_lens, int32_t* q_start, int32_t* num_seqs,
                              int32_t* scratch, int32_t* err_flag, ir_stream_t stream);

/* ---------------------------------------------------------- peer exchange
 *
 * The KV-chunk split over the GPUs of one node (one process per GPU) without
 * a collective library call: in one kernel, every rank's (o, lse) partial
 * (ir_paged_decode_lse) is stored over NVLink into every peer's exchange
 * buffer in 16-byte chunks that carry the call's flag, and each rank merges
 * the world's partials as soon as their flags arrive (ir_lse_merge's
 * arithmetic, in rank order, so all ranks write identical rows). No reference
 * counterpart: infrared is single-GPU. Buffers come from ir_peer_alloc
 * (zeroed) and are mapped into the other processes with ir_peer_handle /
 * ir_peer_open; bufs[] lists all world buffers as seen by the calling
 * process, bufs[rank] being its own. Every rank allocates the same number of
 * bytes (ir_peer_exchange_bytes for the largest batch * num_heads and the
 * head_dim it will use) and passes that size as buffer_bytes: rows are laid
 * out by that capacity, so later calls may use fewer rows (a smaller batch)
 * and a call with more rows than the buffers hold is refused. Every rank must
 * make the same sequence of calls with the same batch, heads and head_dim on
 * one stream; the calls may be captured in a CUDA graph. A peer that stops
 * calling makes the waits run out after 2 s with IR_DEVERR_TIMEOUT, after
 * which the buffers must be allocated anew.
 */
#define IR_PEER_HANDLE_BYTES 64
int ir_peer_alloc(size_t bytes, void** ptr);
int ir_peer_free(void* ptr);
int ir_peer_handle(const void* ptr, void* handle /* IR_PEER_HANDLE_BYTES */);
int ir_peer_open(const void* handle, void** ptr);
int ir_peer_close(void* ptr);
/* Exchange buffer bytes for world ranks, rows = batch * heads, head_dim. */
size_t ir_peer_exchange_bytes(int world, int rows, int head_dim);
/* o [batch * num_heads, head_dim] fp32 (16-byte aligned) and lse
 * [batch * num_heads] fp32 of this rank in; out [batch, num_heads, head_dim]
 * (row stride out_stride, dtype) = all ranks' partials of this call merged.
 * head_dim a multiple of 4 up to 128, world 1..8; buffer_bytes = the size
 * every rank's exchange buffer was allocated with. */
int ir_peer_exchange(void* out, int64_t out_stride, const float* o, const float* lse,
                     void* const* bufs, size_t buffer_bytes, int world, int rank, int batch,
                     int num_heads, int head_dim, int dtype, int32_t* err_flag,
                     ir_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* INFRARED_B200_H_ */
