// K/V pool scatter (cache write), gather, and block-metadata derivation.
//
// Rows are moved in 16-byte vectors when every row start is 16-byte aligned
// (the usual case: [Hkv, D] rows of 512 B - 1 KB), else element by element.
// Each thread moves one vector of one row of K and the same vector of V, so
// a warp writes 512 contiguous bytes of a pool row.
#include "common.cuh"
#include "kernels.h"

namespace irb {

namespace {

template <typename V>
__global__ void cache_write_kernel(const V* __restrict__ k,
                                   const V* __restrict__ v, int64_t k_stride,
                                   int64_t v_stride, V* __restrict__ kp,
                                   V* __restrict__ vp,
                                   const int64_t* __restrict__ slots,
                                   int64_t n, int row_vecs, int64_t num_slots,
                                   int32_t* err) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * row_vecs) return;
  const int64_t tok = i / row_vecs;
  const int c = static_cast<int>(i - tok * row_vecs);
  const int64_t s = slots[tok];
  if (s < 0) return;  // padding row
  if (s >= num_slots) {
    if (c == 0) set_err(err, IR_DEVERR_SLOT);
    return;
  }
  kp[s * row_vecs + c] = k[tok * k_stride + c];
  vp[s * row_vecs + c] = v[tok * v_stride + c];
}

template <typename V>
__global__ void cache_gather_kernel(V* __restrict__ out,
                                    const V* __restrict__ pool,
                                    const int64_t* __restrict__ slots,
                                    int64_t n, int row_vecs, int64_t num_slots,
                                    int32_t* err) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n * row_vecs) return;
  const int64_t r = i / row_vecs;
  const int c = static_cast<int>(i - r * row_vecs);
  const int64_t s = slots[r];
  if (s < 0 || s >= num_slots) {
    if (c == 0) set_err(err, IR_DEVERR_SLOT);
    out[i] = V{};
    return;
  }
  out[i] = pool[s * row_vecs + c];
}

// Mask element is "allowed" iff it is +0 or -0 (any float width).
__device__ __forceinline__ bool mask_zero(const void* mask, int elem_bytes,
                                          int64_t idx) {
  if (elem_bytes == 4)
    return (reinterpret_cast<const uint32_t*>(mask)[idx] & 0x7fffffffu) == 0u;
  return (reinterpret_cast<const uint16_t*>(mask)[idx] & 0x7fffu) == 0u;
}

__global__ void derive_metadata_kernel(const int64_t* __restrict__ gs,
                                       int64_t gs_stride,
                                       const void* __restrict__ mask,
                                       int64_t mask_stride, int elem_bytes,
                                       int64_t T, int bs,
                                       int32_t* __restrict__ bt,
                                       int64_t bt_stride,
                                       int32_t* __restrict__ ctx_out,
                                       int32_t* err) {
  const int b = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t* row = gs + b * gs_stride;
  __shared__ int64_t s_count[32], s_first[32];
  int64_t count = 0, first_nz = T;
  for (int64_t t = tid; t < T; t += blockDim.x) {
    if (mask_zero(mask, elem_bytes, b * mask_stride + t))
      ++count;
    else if (t < first_nz)
      first_nz = t;
  }
  for (int o = 16; o > 0; o >>= 1) {
    count += __shfl_xor_sync(0xffffffffu, count, o);
    first_nz = min(first_nz, __shfl_xor_sync(0xffffffffu, first_nz, o));
  }
  const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    s_count[warp] = count;
    s_first[warp] = first_nz;
  }
  __syncthreads();
  count = 0;
  first_nz = T;
  for (int w = 0; w < nw; ++w) {
    count += s_count[w];
    first_nz = min(first_nz, s_first[w]);
  }
  // a decode mask is a prefix of zeros: the first blocked column is `count`
  if (tid == 0 && first_nz < count) set_err(err, IR_DEVERR_MASK);
  const int64_t ctx = count;
  if (tid == 0) ctx_out[b] = static_cast<int32_t>(ctx);
  const int64_t ncols = (T + bs - 1) / bs;
  const int64_t nblk = (ctx + bs - 1) / bs;
  bool bad = false;
  for (int64_t j = tid; j < ncols; j += blockDim.x) {
    int32_t id = 0;
    if (j < nblk) {
      const int64_t s0 = row[j * bs];
      if (s0 < 0 || s0 % bs != 0 || s0 / bs > INT32_MAX) bad = true;
      id = static_cast<int32_t>(s0 / bs);
    }
    bt[b * bt_stride + j] = id;
  }
  for (int64_t t = tid; t < ctx; t += blockDim.x) {
    const int64_t s0 = row[(t / bs) * bs];
    if (row[t] != (s0 / bs) * bs + t % bs) bad = true;
  }
  if (bad) set_err(err, IR_DEVERR_NOT_BLOCKED);
}

// Fixed-shape decode inputs for a CUDA-graph bucket, one row per block.x:
// row i describes sequence j = (i < batch ? i : 0) (pad rows repeat row 0).
__global__ void build_decode_inputs_kernel(const int32_t* __restrict__ bt, int64_t bt_stride,
                                           const int32_t* __restrict__ num_cached,
                                           const int64_t* __restrict__ last_tokens,
                                           int batch, int64_t t_max, int bs,
                                           int64_t* __restrict__ ids,
                                           int64_t* __restrict__ positions,
                                           int64_t* __restrict__ write_slots,
                                           int64_t* __restrict__ gather_slots, void* mask,
                                           int mask_bytes, uint32_t min_bits) {
  const int i = blockIdx.x;
  const int j = i < batch ? i : 0;
  const int32_t* row = bt + j * bt_stride;
  const int64_t nc = num_cached[j];
  const int64_t ctx = nc + 1;
  const int64_t t = static_cast<int64_t>(blockIdx.y) * blockDim.x + threadIdx.x;
  if (t == 0) {
    ids[i] = last_tokens[j];
    positions[i] = nc;
    write_slots[i] = static_cast<int64_t>(row[nc / bs]) * bs + nc % bs;
  }
  if (t >= t_max) return;
  const bool valid = t < ctx;
  gather_slots[i * t_max + t] = valid ? static_cast<int64_t>(row[t / bs]) * bs + t % bs : 0;
  if (mask_bytes == 4)
    reinterpret_cast<uint32_t*>(mask)[i * t_max + t] = valid ? 0u : min_bits;
  else
    reinterpret_cast<uint16_t*>(mask)[i * t_max + t] =
        static_cast<uint16_t>(valid ? 0u : min_bits);
}

// Per query row of a packed prefill: the row's sequence (largest s with
// q_start[s] <= t), its context (position + 1) and a copy of the sequence's
// block-table row, so that every row can be decoded as its own sequence.
__global__ void prefill_rows_kernel(const int32_t* __restrict__ bt, int64_t bt_stride,
                                    const int32_t* __restrict__ ctx,
                                    const int32_t* __restrict__ q_start, int S, int max_blocks,
                                    int max_ctx, int32_t* __restrict__ row_bt,
                                    int32_t* __restrict__ row_ctx, int32_t* err) {
  const int t = blockIdx.x;
  __shared__ int s_seq;
  if (threadIdx.x == 0) {
    int lo = 0, hi = S - 1, found = -1;
    while (lo <= hi) {
      const int mid = (lo + hi) >> 1;
      if (q_start[mid] <= t) {
        found = mid;
        lo = mid + 1;
      } else {
        hi = mid - 1;
      }
    }
    int c = 0;
    if (found >= 0 && t < q_start[found + 1]) {
      const int ql = q_start[found + 1] - q_start[found];
      const int cs = ctx[found];
      if (cs < ql || cs > max_ctx) {
        set_err(err, IR_DEVERR_CONTEXT_LEN);
      } else {
        c = cs - ql + (t - q_start[found]) + 1;
      }
    } else {
      found = -1;
    }
    row_ctx[t] = c;
    s_seq = found;
  }
  __syncthreads();
  const int sq = s_seq;
  for (int j = threadIdx.x; j < max_blocks; j += blockDim.x)
    row_bt[static_cast<int64_t>(t) * max_blocks + j] =
        sq >= 0 ? bt[static_cast<int64_t>(sq) * bt_stride + j] : 0;
}

// ---- packed prefill frames (Sq > 1): (gather_slots, mask) -> block tables
//
// infrared's mixed step gathers every sequence's history into one key axis
// and masks each query row to its own sequence's causal prefix
// (infrared/model/inputs.py:64-94); its single-prompt prefill is the same
// with one sequence (:38-61). Row i of such a mask allows exactly one
// contiguous key range [lo_i, lo_i + cnt_i); consecutive rows with the same lo
// form a sequence whose cnt grows by one per row; its history is the key
// range of its last row, block-structured from lo.

// Per query row: first allowed key column and the number of allowed columns
// (flags MASK when they are not one contiguous range).
__global__ void varlen_rows_kernel(const void* __restrict__ mask, int64_t mask_stride,
                                   int elem_bytes, int64_t K, int32_t* __restrict__ lo,
                                   int32_t* __restrict__ cnt, int32_t* err) {
  const int64_t i = blockIdx.x;
  const int tid = threadIdx.x;
  __shared__ int64_t s_cnt[32], s_min[32], s_max[32];
  int64_t c = 0, mn = K, mx = -1;
  for (int64_t t = tid; t < K; t += blockDim.x) {
    if (mask_zero(mask, elem_bytes, i * mask_stride + t)) {
      ++c;
      mn = t < mn ? t : mn;
      mx = t > mx ? t : mx;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    c += __shfl_xor_sync(0xffffffffu, c, o);
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    s_cnt[warp] = c;
    s_min[warp] = mn;
    s_max[warp] = mx;
  }
  __syncthreads();
  if (tid == 0) {
    c = 0;
    mn = K;
    mx = -1;
    for (int w = 0; w < nw; ++w) {
      c += s_cnt[w];
      mn = min(mn, s_min[w]);
      mx = max(mx, s_max[w]);
    }
    if (c == 0 || mx - mn + 1 != c) set_err(err, IR_DEVERR_MASK);
    lo[i] = static_cast<int32_t>(c == 0 ? 0 : mn);
    cnt[i] = static_cast<int32_t>(c);
  }
}

// One block: sequence boundaries (rows whose lo differs from the previous
// row's), q_start, the history length of each sequence (cnt of its last
// row) and its first key column; checks that cnt grows by one per row.
__global__ void varlen_seqs_kernel(const int32_t* __restrict__ lo, const int32_t* __restrict__ cnt,
                                   int Q, int32_t* __restrict__ q_start, int32_t* __restrict__ ctx,
                                   int32_t* __restrict__ lo_seq, int32_t* __restrict__ nseq,
                                   int32_t* err) {
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < Q; base += blockDim.x) {
    const int i = base + tid;
    const bool valid = i < Q;
    const bool start = valid && (i == 0 || lo[i] != lo[i - 1]);
    if (valid && !start && cnt[i] != cnt[i - 1] + 1) set_err(err, IR_DEVERR_MASK);
    // block-wide inclusive scan of the start flags
    int v = start ? 1 : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (lane == 31) s_warp[warp] = v;
    __syncthreads();
    if (warp == 0) {
      int w = lane < nw ? s_warp[lane] : 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nw) s_warp[lane] = w;
    }
    __syncthreads();
    const int incl = v + (warp > 0 ? s_warp[warp - 1] : 0) + s_carry;
    const int seq = incl - 1;  // sequence of row i
    if (start) {
      q_start[seq] = i;
      lo_seq[seq] = lo[i];
    }
    if (valid && (i == Q - 1 || lo[i + 1] != lo[i])) ctx[seq] = cnt[i];
    __syncthreads();
    if (tid == blockDim.x - 1) s_carry = incl;
    __syncthreads();
  }
  if (tid == 0) {
    q_start[s_carry] = Q;
    *nseq = s_carry;
  }
}

// Block table of sequence blockIdx.x from its key range of the gathered
// slots; flags NOT_BLOCKED when the range is not block-structured.
__global__ void varlen_tables_kernel(const int64_t* __restrict__ gs, const int32_t* __restrict__ lo_seq,
                                     const int32_t* __restrict__ ctx, const int32_t* __restrict__ nseq,
                                     int bs, int max_blocks, int32_t* __restrict__ bt,
                                     int32_t* err) {
  const int sq = blockIdx.x;
  if (sq >= *nseq) return;
  const int64_t base = lo_seq[sq];
  const int c = ctx[sq];
  const int nb = (c + bs - 1) / bs;
  if (nb > max_blocks) {
    if (threadIdx.x == 0) set_err(err, IR_DEVERR_CONTEXT_LEN);
    return;
  }
  bool bad = false;
  for (int j = threadIdx.x; j < max_blocks; j += blockDim.x) {
    int32_t id = 0;
    if (j < nb) {
      const int64_t s0 = gs[base + static_cast<int64_t>(j) * bs];
      if (s0 < 0 || s0 % bs != 0 || s0 / bs > INT32_MAX) bad = true;
      id = static_cast<int32_t>(s0 / bs);
    }
    bt[static_cast<int64_t>(sq) * max_blocks + j] = id;
  }
  for (int t = threadIdx.x; t < c; t += blockDim.x) {
    const int64_t s0 = gs[base + (t / bs) * bs];
    if (gs[base + t] != (s0 / bs) * bs + t % bs) bad = true;
  }
  if (bad) set_err(err, IR_DEVERR_NOT_BLOCKED);
}

int grid_for(int64_t work, int threads) {
  return static_cast<int>((work + threads - 1) / threads);
}

}  // namespace

int launch_cache_write(const void* k, const void* v, int64_t k_stride,
                       int64_t v_stride, void* k_pool, void* v_pool,
                       const int64_t* slots, int64_t n, int row_elems,
                       int64_t num_slots, int elem_bytes, int32_t* err,
                       cudaStream_t stream) {
  if (n == 0) return 0;
  const int row_bytes = row_elems * elem_bytes;
  const bool vec = (row_bytes % 16 == 0) && ((k_stride * elem_bytes) % 16 == 0) &&
                   ((v_stride * elem_bytes) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(k) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(v) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(k_pool) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(v_pool) % 16 == 0);
  const int threads = 256;
  if (vec) {
    const int rv = row_bytes / 16;
    const int64_t ks = k_stride * elem_bytes / 16, vs = v_stride * elem_bytes / 16;
    cache_write_kernel<uint4><<<grid_for(n * rv, threads), threads, 0, stream>>>(
        static_cast<const uint4*>(k), static_cast<const uint4*>(v), ks, vs,
        static_cast<uint4*>(k_pool), static_cast<uint4*>(v_pool), slots, n, rv,
        num_slots, err);
  } else if (elem_bytes == 4) {
    cache_write_kernel<uint32_t><<<grid_for(n * row_elems, threads), threads, 0, stream>>>(
        static_cast<const uint32_t*>(k), static_cast<const uint32_t*>(v), k_stride,
        v_stride, static_cast<uint32_t*>(k_pool), static_cast<uint32_t*>(v_pool),
        slots, n, row_elems, num_slots, err);
  } else {
    cache_write_kernel<uint16_t><<<grid_for(n * row_elems, threads), threads, 0, stream>>>(
        static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v), k_stride,
        v_stride, static_cast<uint16_t*>(k_pool), static_cast<uint16_t*>(v_pool),
        slots, n, row_elems, num_slots, err);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_cache_gather(void* out, const void* pool, const int64_t* slots,
                        int64_t n, int row_elems, int64_t num_slots,
                        int elem_bytes, int32_t* err, cudaStream_t stream) {
  if (n == 0) return 0;
  const int row_bytes = row_elems * elem_bytes;
  const int threads = 256;
  const bool vec = (row_bytes % 16 == 0) && (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(pool) % 16 == 0);
  if (vec) {
    const int rv = row_bytes / 16;
    cache_gather_kernel<uint4><<<grid_for(n * rv, threads), threads, 0, stream>>>(
        static_cast<uint4*>(out), static_cast<const uint4*>(pool), slots, n, rv,
        num_slots, err);
  } else if (elem_bytes == 4) {
    cache_gather_kernel<uint32_t><<<grid_for(n * row_elems, threads), threads, 0, stream>>>(
        static_cast<uint32_t*>(out), static_cast<const uint32_t*>(pool), slots, n,
        row_elems, num_slots, err);
  } else {
    cache_gather_kernel<uint16_t><<<grid_for(n * row_elems, threads), threads, 0, stream>>>(
        static_cast<uint16_t*>(out), static_cast<const uint16_t*>(pool), slots, n,
        row_elems, num_slots, err);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_build_decode_inputs(const int32_t* bt, int64_t bt_stride,
                               const int32_t* num_cached, const int64_t* last_tokens,
                               int batch, int bucket, int64_t t_max, int bs, int64_t* ids,
                               int64_t* positions, int64_t* write_slots,
                               int64_t* gather_slots, void* mask, int mask_bytes,
                               uint32_t min_bits, cudaStream_t stream) {
  if (bucket == 0) return 0;
  dim3 grid(bucket, static_cast<unsigned>((t_max + 255) / 256));
  build_decode_inputs_kernel<<<grid, 256, 0, stream>>>(bt, bt_stride, num_cached, last_tokens,
                                                       batch, t_max, bs, ids, positions,
                                                       write_slots, gather_slots, mask,
                                                       mask_bytes, min_bits);
  return static_cast<int>(cudaGetLastError());
}

int launch_prefill_rows(const int32_t* bt, int64_t bt_stride, const int32_t* ctx,
                        const int32_t* q_start, int S, int total_q, int max_blocks, int max_ctx,
                        int32_t* row_bt, int32_t* row_ctx, int32_t* err, cudaStream_t stream) {
  if (total_q == 0) return 0;
  prefill_rows_kernel<<<total_q, 128, 0, stream>>>(bt, bt_stride, ctx, q_start, S, max_blocks,
                                                   max_ctx, row_bt, row_ctx, err);
  return static_cast<int>(cudaGetLastError());
}

int launch_derive_varlen(const int64_t* gs, const void* mask, int64_t mask_stride,
                         int mask_elem_bytes, int Q, int64_t K, int bs, int max_blocks,
                         int32_t* bt, int32_t* ctx, int32_t* q_start, int32_t* nseq,
                         int32_t* scratch, int32_t* err, cudaStream_t stream) {
  if (Q == 0) {
    cudaError_t e = cudaMemsetAsync(nseq, 0, 4, stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(q_start, 0, 4, stream);
    return static_cast<int>(e);
  }
  int32_t* lo = scratch;
  int32_t* cnt = scratch + Q;
  int32_t* lo_seq = scratch + 2 * static_cast<int64_t>(Q);
  varlen_rows_kernel<<<Q, 256, 0, stream>>>(mask, mask_stride, mask_elem_bytes, K, lo, cnt, err);
  varlen_seqs_kernel<<<1, 1024, 0, stream>>>(lo, cnt, Q, q_start, ctx, lo_seq, nseq, err);
  varlen_tables_kernel<<<Q, 128, 0, stream>>>(gs, lo_seq, ctx, nseq, bs, max_blocks, bt, err);
  return static_cast<int>(cudaGetLastError());
}

int launch_derive_metadata(const int64_t* gs, int64_t gs_stride,
                           const void* mask, int64_t mask_stride,
                           int mask_elem_bytes, int B, int64_t T, int bs,
                           int32_t* bt, int64_t bt_stride, int32_t* ctx,
                           int32_t* err, cudaStream_t stream) {
  if (B == 0) return 0;
  derive_metadata_kernel<<<B, 256, 0, stream>>>(gs, gs_stride, mask, mask_stride,
                                                mask_elem_bytes, T, bs, bt,
                                                bt_stride, ctx, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace irb
