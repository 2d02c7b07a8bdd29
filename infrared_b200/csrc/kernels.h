// Host-side launchers of the infrared_b200 kernels (internal interface
// between the C ABI in capi.cu and the kernel translation units).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace irb {

struct DecodeArgs;

// Packed-query paged prefill (prefill_tc.cu): sequence s owns query rows
// [q_start[s], q_start[s+1]) = its last q_len positions of context_lens[s].
struct PrefillArgs {
  const void* q;  // [total_q, H, D] rows with row stride q_stride
  int64_t q_stride;
  void* out;  // same layout, out_stride
  int64_t out_stride;
  const int32_t* block_tables;  // [S, max_blocks] with bt_stride
  int64_t bt_stride;
  const int32_t* context_lens;  // [S]
  const int32_t* q_start;       // [S + 1]
  int S, total_q, H, Hkv, n_rep, D, bs, max_blocks;
  int64_t num_slots, num_blocks;
  float scale_log2;
  int32_t* err;
};

// tcgen05 kernel: 16-bit dtypes, D in {64, 128}, block size a power of two
// >= 8; tmq views q as (D, H, total_q), tmk/tmv the pools as (D, Hkv, slots)
// with boxes {64, 1, 128} (q) and {64, 1, min(bs, 128)} (128-byte swizzle).
// pair: the CTA-pair form (D = 128; cta_group::2, 256-row items), whose K
// map has boxes {64, 1, min(bs, 64)}.
int launch_prefill_tc(const CUtensorMap& tmq, const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const PrefillArgs& a, int dtype, int sm_count, bool pair,
                      cudaStream_t stream);

// kv_proj.cu: K/V projection of M new tokens (x [M, K], W_k / W_v [Hkv*D, K]
// row-major, K % 64 == 0) with bias, RoPE on K and the pool write in the
// epilogue; tmx views x as (K, M), tmwk / tmwv the weights as (K, Hkv*D),
// boxes {64, 128} and {64, D}, 128-byte swizzle.
struct KvProjArgs {
  int M, K, Hkv, D;
  const void* bias_k;  // [Hkv * D] of the dtype, or null
  const void* bias_v;
  const float* cos;    // [M, D] rows with rope_stride, or null (no RoPE)
  const float* sin;
  int64_t rope_stride;
  const int64_t* slots;  // [M]
  void* k_pool;          // [num_slots, Hkv, D]
  void* v_pool;
  int64_t num_slots;
  int32_t* err;
};
int launch_kv_proj(const CUtensorMap& tmx, const CUtensorMap& tmwk, const CUtensorMap& tmwv,
                   const KvProjArgs& a, int dtype, cudaStream_t s);

// peer_exchange.cu: KV-chunk partials stored into every GPU of the node
// (buffers mapped with CUDA IPC) in a flagged 16-byte chunk format and merged,
// in one kernel; see the file header for the buffer layout and the protocol.
struct PeerArgs {
  uint8_t* bufs[8];  // every rank's exchange buffer as mapped in this process
  int world, rank;
  int rows, D;       // rows = batch * heads of this call
  int cap;           // rows the buffers are laid out for (from their size)
  int sms;           // SM count of this device (bounds the grid)
  int32_t* err;
};
size_t peer_exchange_bytes(int world, int rows, int D);
int64_t peer_exchange_capacity(size_t bytes, int world, int D);
int peer_exchange_grid(int64_t cap, int sms);
int launch_peer_exchange(void* out, int64_t out_stride, const float* o, const float* lse, int H,
                         int dtype, const PeerArgs& p, cudaStream_t s);

// decode_tma.cu: 16-bit pools, D in {64, 128}, group <= 8, bs == 8 or bs % 16 == 0.
// One CTA covers tma_head_group(Hkv) kv heads; one_box selects the 4-D
// (one copy per tile side) or the 3-D (one copy per head and half) map.
int tma_head_group(int num_kv_heads);
int launch_decode_tma(const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const DecodeArgs& a, int dtype, int one_box, int stall,
                      cudaStream_t stream);
int decode_tma_occupancy(int dtype, int D, int Hkv, int bs);

// decode_generic.cu: any dtype, D in {64, 128}, group <= 16, any block size
int launch_decode_generic(const DecodeArgs& a, int dtype, cudaStream_t stream);
int decode_generic_occupancy(int dtype, int D);

// merges (decode_generic.cu): the pieces of sequences split across CTAs
// (programmatic dependent launch behind the decode kernel), and partials of
// KV ranges computed elsewhere (e.g. other GPUs)
int launch_split_merge(const DecodeArgs& a, int dtype, cudaStream_t stream);
int launch_lse_merge(void* out, int64_t out_stride, const float* o_parts,
                     int64_t o_part_stride, const float* lse_parts,
                     int64_t lse_part_stride, int P, int B, int H, int D,
                     int dtype, cudaStream_t stream);

// cache_ops.cu
int launch_cache_write(const void* k, const void* v, int64_t k_stride,
                       int64_t v_stride, void* k_pool, void* v_pool,
                       const int64_t* slots, int64_t n, int row_elems,
                       int64_t num_slots, int elem_bytes, int32_t* err,
                       cudaStream_t stream);
int launch_cache_gather(void* out, const void* pool, const int64_t* slots,
                        int64_t n, int row_elems, int64_t num_slots,
                        int elem_bytes, int32_t* err, cudaStream_t stream);
int launch_build_decode_inputs(const int32_t* bt, int64_t bt_stride,
                               const int32_t* num_cached, const int64_t* last_tokens,
                               int batch, int bucket, int64_t t_max, int bs, int64_t* ids,
                               int64_t* positions, int64_t* write_slots,
                               int64_t* gather_slots, void* mask, int mask_bytes,
                               uint32_t min_bits, cudaStream_t stream);
int launch_prefill_rows(const int32_t* bt, int64_t bt_stride, const int32_t* ctx,
                        const int32_t* q_start, int S, int total_q, int max_blocks, int max_ctx,
                        int32_t* row_bt, int32_t* row_ctx, int32_t* err, cudaStream_t stream);
int launch_derive_varlen(const int64_t* gs, const void* mask, int64_t mask_stride,
                         int mask_elem_bytes, int Q, int64_t K, int bs, int max_blocks,
                         int32_t* bt, int32_t* ctx, int32_t* q_start, int32_t* nseq,
                         int32_t* scratch, int32_t* err, cudaStream_t stream);
int launch_derive_metadata(const int64_t* gs, int64_t gs_stride,
                           const void* mask, int64_t mask_stride,
                           int mask_elem_bytes, int B, int64_t T, int bs,
                           int32_t* bt, int64_t bt_stride, int32_t* ctx,
                           int32_t* err, cudaStream_t stream);

}  // namespace irb
