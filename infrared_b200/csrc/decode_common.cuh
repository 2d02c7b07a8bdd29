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
//
// Dynamic tail (TMA kernel, DecodeArgs::dyn): the tile axis is cut into
// units instead — Gs static units (equal shares of the first F tiles, one per
// CTA) followed by U small dynamic units covering tiles [F, T), which the
// CTAs claim from a counter in the workspace header once their static unit
// is streamed. SMs stream at slightly different, randomly varying rates, so
// with static shares alone the last CTA finishes several microseconds after
// the median one; claimed units let the fast CTAs take more of the tail. A
// unit plays the part of a share: pieces sit in slot u + b, and the merge
// finds a sequence's units with unit_of(), a function of T alone, so the
// result does not depend on which CTA took which unit. The dynamic tiles lie
// in the last kDynSeqs sequences (their prefixes fit in shared memory for the
// claim's lookup). The counter pair {claims, CTAs done} of each kv-head group
// is zero at the start of every call: the caller zeroes the header once when
// it allocates the workspace, and the last CTA of every call (every exit
// path counts itself done) sets both back to zero.
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
  int dyn;           // 1: dynamic tail units (ws_ctr zero at the start of the call)
  int inline_merge;  // 1: short rows merged in the decode kernel (ws_seq zero at the start)
  int zeroed;        // dyn || inline_merge: the header counters are in use
  // workspace
  uint32_t* ws_ctr;    // [kv-head groups][2] {claims, CTAs done} of the dynamic tail
  uint32_t* ws_seq;    // [Hkv, B] pieces of a (kv head, sequence) row written so far
  int64_t* ws_prefix;  // [B + 1] tile prefix (written by the first CTA of kv head 0)
  int64_t ws_slots;    // partial slots per kv head: G (+ kDynUnitsPerCta * G) + B
  float* ws_lse;       // [Hkv, ws_slots, n_rep] log2-sum-exp of partials
  float* ws_o;         // [Hkv, ws_slots, n_rep, D] normalised partials
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

// Dynamic tail tuning: the share of the tiles handed out as claimed units,
// the smallest unit, the cap on the unit count (per CTA of the grid), the
// fewest tiles per CTA for which the tail is split at all, and the number of
// trailing sequences the dynamic tiles may lie in.
constexpr int kDynPct = 15;
constexpr int kDynUnitTiles = 4;
constexpr int kDynUnitsPerCta = 2;
constexpr int kDynMinTilesPerCta = 8;
constexpr int kDynSeqs = 32;
// In-kernel merge (DecodeArgs::inline_merge): a row split into at most this
// many pieces is merged by the warp that writes its last piece; longer rows
// are left to the merge kernel.
constexpr int kInlineMax = 4;

struct UnitPlan {
  int64_t F;    // static tiles [0, F), cut into Gs equal shares
  int64_t dyn;  // dynamic tiles [F, F + dyn), cut into U units
  int Gs;       // static units (one per CTA g < Gs)
  int U;        // dynamic units
};

// The unit plan of a call with T tiles on G CTAs per kv-head group; p_tail =
// tile prefix of sequence max(B - kDynSeqs, 0). dyn_on = 0 gives the static
// plan (Gs = min(T, G) equal shares, no dynamic units).
__host__ __device__ __forceinline__ UnitPlan unit_plan(int64_t T, int G, int dyn_on,
                                                       int64_t p_tail) {
  UnitPlan u{T, 0, 0, 0};
  if (dyn_on && T >= static_cast<int64_t>(kDynMinTilesPerCta) * G) {
    int64_t F = T - T * kDynPct / 100;
    if (F < p_tail) F = p_tail;
    const int64_t d = T - F;
    if (d > 0) {
      const int64_t n = (d + kDynUnitTiles - 1) / kDynUnitTiles;
      const int64_t cap = static_cast<int64_t>(kDynUnitsPerCta) * G;
      u.U = static_cast<int>(n < cap ? n : cap);
      u.F = F;
      u.dyn = d;
    }
  }
  u.Gs = u.F < G ? static_cast<int>(u.F) : G;
  return u;
}

// First tile of unit u (0 <= u <= Gs + U; u = Gs + U gives T).
__device__ __forceinline__ int64_t unit_start(const UnitPlan& p, int64_t u) {
  return u < p.Gs ? share_start(u, p.F, p.Gs)
                  : p.F + share_start(u - p.Gs, p.dyn, p.U);
}

// Unit holding tile t (0 <= t < T).
__device__ __forceinline__ int unit_of(const UnitPlan& p, int64_t t) {
  return t < p.F ? share_of(t, p.F, p.Gs) : p.Gs + share_of(t - p.F, p.dyn, p.U);
}

struct RangeInfo {
  int64_t total;    // T
  int64_t start;    // first tile of this CTA's static unit
  int64_t end;      // one past its last tile
  int64_t p_first;  // prefix of b_first
  int b_first;      // sequence holding tile `start`
  int G;            // static units (<= DecodeArgs::G)
  UnitPlan plan;
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

// Prefixes and context lengths of the last kDynSeqs sequences (tailp[i] =
// prefix of sequence B0 + i, tailp[B - B0] = T, tailc[i] = its clamped
// context length; B0 = max(B - kDynSeqs, 0)), computed by warp 0 from the
// context lengths once T is known, so that the producer resolves a dynamic
// unit without global loads. Warp 0 only; the caller synchronises before the
// arrays are read.
__device__ __forceinline__ void tail_prefixes(const DecodeArgs& a, int64_t total,
                                              int64_t* tailp, int* tailc) {
  const int lane = threadIdx.x & 31;
  const int b0 = a.B > kDynSeqs ? a.B - kDynSeqs : 0;
  const int nt = a.B - b0;
  const int c = lane < nt ? clamp_ctx(a.context_lens[b0 + lane], a) : 0;
  const int n = (c + kTile - 1) / kTile;
  // suffix sum from this lane to the last: inclusive scan of the reversed lanes
  int suf = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, suf, o);
    if (lane + o < 32) suf += y;
  }
  if (lane < nt) {
    tailp[lane] = total - suf;
    tailc[lane] = c;
  }
  if (lane == 0) tailp[nt] = total;
}

// Find this CTA's share (its static unit under a dynamic plan). All NT
// threads must call it. The CTA streams kv heads [kv0, kv0 + nkv). The first
// CTA of kv head 0 publishes the tile prefix to the workspace for the merge
// kernel; CTAs with g == 0 write the rows of sequences with no context (no
// CTA streams them). With a.dyn, tailp / tailc (shared memory, kDynSeqs + 1
// and kDynSeqs entries) receive the prefixes and context lengths of the
// sequences the dynamic tiles lie in.
template <int NT, typename T>
__device__ void find_share(const DecodeArgs& a, int g, int kv0, int nkv,
                           RangeInfo* ri, int64_t* sm_scan, int64_t* tailp = nullptr,
                           int* tailc = nullptr) {
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
  // the unit plan once T is known (tail prefixes first when dynamic)
  auto make_plan = [&](int64_t total) {
    const bool dyn = a.dyn && tailp != nullptr;
    if (dyn && tid < 32) tail_prefixes(a, total, tailp, tailc);
    if (dyn) __syncthreads();
    return unit_plan(total, a.G, dyn ? 1 : 0, dyn ? tailp[0] : 0);
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
    const UnitPlan up = make_plan(total);
    const int G = up.Gs;
    const int64_t start = g < G ? share_start(g, up.F, G) : total;
    const int64_t end = g < G ? share_start(g + 1, up.F, G) : total;
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
      ri->plan = up;
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
  const UnitPlan up = make_plan(total);
  const int G = up.Gs;
  const int64_t start = g < G ? share_start(g, up.F, G) : total;
  const int64_t end = g < G ? share_start(g + 1, up.F, G) : total;
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
    ri->plan = up;
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
    const int64_t slot = static_cast<int64_t>(kvh) * a.ws_slots + g + b;
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
