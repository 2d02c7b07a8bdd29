// Work partition and output conventions shared by the decode kernels.
//
// Units of work are 16-token "tiles" of one (sequence, kv-head) history:
// sequence b has n_b = ceil(ctx_b / 16) tiles. For each kv head the tiles of
// all sequences are laid end to end (prefix P_b = sum_{b' < b} n_b', total
// T) and cut into G equal shares: CTA g of that kv head streams tiles
// [start(g), start(g+1)) with start(g) = floor(g * T / G). A share may cover
// the tail of one sequence, several whole sequences and the head of another;
// each (CTA, sequence) piece is a "segment". A segment that is a whole
// sequence writes the final row; any other segment writes a normalised fp32
// partial and its log2-sum-exp into workspace slot g + b (unique: along the
// monotone path of (g, b) pieces g + b strictly increases). The merge kernel,
// launched right behind the decode kernel (programmatic dependent launch),
// combines the pieces of every sequence that spans several CTAs in share
// order, so results do not depend on scheduling.
#pragma once

#include "common.cuh"

namespace irb {

constexpr int kTile = 16;  // tokens per tile

struct DecodeArgs {
  const void* q;
  int64_t q_stride;
  void* out;  // final output (dtype T) [B, H, D] with out_stride
  int64_t out_stride;
  float* lse_o;    // LSE mode: o [B, H, D] fp32 contiguous
  float* lse_out;  // LSE mode: lse [B, H] natural log
  int lse_mode;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* context_lens;
  int B, H, Hkv, n_rep, D, bs, max_blocks;
  int64_t num_slots, num_blocks;
  float scale_log2;  // scale * log2(e)
  int G;             // CTAs per kv head
  // workspace
  int64_t* ws_prefix;  // [B + 1] tile prefix (written by the first CTA of kv head 0)
  float* ws_lse;       // [Hkv, G + B, n_rep] log2-sum-exp of partials
  float* ws_o;         // [Hkv, G + B, n_rep, D] normalised partials
  // pools (generic kernel reads them directly; fused write stores into them)
  const void* k_pool;
  const void* v_pool;
  // fused cache write of this step's K/V (null when not fused)
  const void* k_new;
  const void* v_new;
  int64_t kv_stride;
  const int64_t* slot_mapping;
  // RoPE applied to q and to the new token's K inside the kernel (null: the
  // inputs are already rotated): fp32 cos/sin rows [B, D] with rope_stride
  const float* rope_cos;
  const float* rope_sin;
  int64_t rope_stride;
  int32_t* err;
};

__device__ __forceinline__ int clamp_ctx(int c, const DecodeArgs& a) {
  const int maxc = a.max_blocks * a.bs;
  return c < 0 ? 0 : (c > maxc ? maxc : c);
}

__device__ __forceinline__ int tiles_of(const DecodeArgs& a, int b) {
  return (clamp_ctx(a.context_lens[b], a) + kTile - 1) / kTile;
}

__device__ __forceinline__ int64_t share_start(int64_t g, int64_t total,
                                               int G) {
  return (g * total) / G;
}

// CTA whose share holds tile t (0 <= t < total).
__device__ __forceinline__ int share_of(int64_t t, int64_t total, int G) {
  return static_cast<int>(((t + 1) * G + total - 1) / total - 1);
}

// Shares actually used: never more CTAs than tiles, so no share is empty.
__device__ __forceinline__ int shares_used(int64_t total, int G) {
  return total < G ? static_cast<int>(total) : G;
}

struct RangeInfo {
  int64_t total;    // T
  int64_t start;    // first tile of this CTA
  int64_t end;      // one past the last tile
  int64_t p_first;  // prefix of b_first
  int b_first;      // sequence holding tile `start`
  int G;            // shares used (<= DecodeArgs::G)
};

// Block-wide exclusive scan of one int64 per thread (NT threads, NT % 32 == 0).
template <int NT>
__device__ __forceinline__ int64_t block_excl_scan(int64_t v, int64_t* sm,
                                                   int64_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sm[warp] = x;
  __syncthreads();
  int64_t before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) {
    const int64_t s = sm[w];
    if (w < warp) before += s;
    all += s;
  }
  __syncthreads();
  *total = all;
  return before + x - v;
}

// Find this CTA's share. All NT threads must call it. The CTA streams kv
// heads [kv0, kv0 + nkv). The first CTA of kv head 0 publishes the tile
// prefix to the workspace for the merge kernel; CTAs with g == 0 write the
// rows of sequences with no context (no CTA streams them).
template <int NT, typename T>
__device__ void find_share(const DecodeArgs& a, int g, int kv0, int nkv,
                           RangeInfo* ri, int64_t* sm_scan) {
  const int tid = threadIdx.x;
  const bool publish = (g == 0 && kv0 == 0);
  auto empty_rows = [&](int b) {
    // empty context: zero rows (and lse = -inf) of this CTA's heads
    for (int i = 0; i < nkv * a.n_rep * a.D; ++i) {
      const int h = kv0 * a.n_rep + i / a.D, d = i % a.D;
      if (a.lse_mode) {
        a.lse_o[(static_cast<int64_t>(b) * a.H + h) * a.D + d] = 0.f;
        if (d == 0) a.lse_out[static_cast<int64_t>(b) * a.H + h] = -INFINITY;
      } else {
        reinterpret_cast<T*>(a.out)[b * a.out_stride + h * a.D + d] = DT<T>::from_f(0.f);
      }
    }
  };
  if (tid == 0) ri->b_first = -1;
  if (a.B <= NT) {
    // one pass: every thread owns one sequence
    const int b = tid;
    int n = 0;
    if (b < a.B) {
      const int c = a.context_lens[b];
      if (c < 0 || c > a.max_blocks * a.bs) set_err(a.err, IR_DEVERR_CONTEXT_LEN);
      n = tiles_of(a, b);
    }
    int64_t total = 0;
    const int64_t p = block_excl_scan<NT>(n, sm_scan, &total);  // synchronises
    const int G = shares_used(total, a.G);
    const int64_t start = g < G ? share_start(g, total, G) : total;
    const int64_t end = g < G ? share_start(g + 1, total, G) : total;
    if (b < a.B) {
      if (publish) a.ws_prefix[b] = p;
      if (n > 0 && p <= start && start < p + n) {
        ri->b_first = b;
        ri->p_first = p;
      }
      if (n == 0 && g == 0) empty_rows(b);
    }
    if (tid == 0) {
      ri->total = total;
      ri->start = start;
      ri->end = end;
      ri->G = G;
      if (publish) a.ws_prefix[a.B] = total;
    }
    __syncthreads();
    return;
  }
  // pass 1: total tiles (and context validation)
  int64_t mine = 0;
  for (int b = tid; b < a.B; b += NT) {
    const int c = a.context_lens[b];
    if (c < 0 || c > a.max_blocks * a.bs) set_err(a.err, IR_DEVERR_CONTEXT_LEN);
    mine += tiles_of(a, b);
  }
  int64_t total = 0;
  block_excl_scan<NT>(mine, sm_scan, &total);
  const int G = shares_used(total, a.G);
  const int64_t start = g < G ? share_start(g, total, G) : total;
  const int64_t end = g < G ? share_start(g + 1, total, G) : total;
  // pass 2: prefix of every sequence; locate `start`
  int64_t running = 0;
  for (int base = 0; base < a.B; base += NT) {
    const int b = base + tid;
    const int n = b < a.B ? tiles_of(a, b) : 0;
    int64_t chunk_total = 0;
    const int64_t p = running + block_excl_scan<NT>(n, sm_scan, &chunk_total);
    if (b < a.B) {
      if (publish) a.ws_prefix[b] = p;
      if (n > 0 && p <= start && start < p + n) {
        ri->b_first = b;
        ri->p_first = p;
      }
      if (n == 0 && g == 0) empty_rows(b);
    }
    running += chunk_total;
  }
  if (tid == 0) {
    ri->total = total;
    ri->start = start;
    ri->end = end;
    ri->G = G;
    if (publish) a.ws_prefix[a.B] = total;
  }
  __syncthreads();
}

// Write one output value of a segment: final row, LSE-mode row or partial.
template <typename T>
__device__ __forceinline__ void write_segment_value(const DecodeArgs& a,
                                                   int kvh, int g, int b,
                                                   bool whole, int n, int d,
                                                   float val, float lse2) {
  const int h = kvh * a.n_rep + n;
  if (whole) {
    if (a.lse_mode) {
      a.lse_o[(static_cast<int64_t>(b) * a.H + h) * a.D + d] = val;
      if (d == 0) a.lse_out[static_cast<int64_t>(b) * a.H + h] = lse2 * kLn2;
    } else {
      reinterpret_cast<T*>(a.out)[b * a.out_stride + static_cast<int64_t>(h) * a.D + d] =
          DT<T>::from_f(val);
    }
  } else {
    const int64_t slot =
        static_cast<int64_t>(kvh) * (a.G + a.B) + g + b;
    a.ws_o[(slot * a.n_rep + n) * a.D + d] = val;
    if (d == 0) a.ws_lse[slot * a.n_rep + n] = lse2;
  }
}

// Shares [glo, glo + parts) hold the pieces of a sequence with tile prefix
// pb and nb tiles.
__device__ __forceinline__ void piece_range(int64_t pb, int64_t nb, int64_t total, int G,
                                            int* glo, int* parts) {
  const int lo = share_of(pb, total, G);
  *glo = lo;
  *parts = share_of(pb + nb - 1, total, G) - lo + 1;
}

// Programmatic dependent launch: let the dependent (merge) grid start
// launching now / wait until the prerequisite (decode) grid has finished and
// its memory is visible. Both are no-ops without a dependent launch.
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_prerequisites() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace irb
