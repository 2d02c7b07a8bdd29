// Paged prefill / mixed-varlen attention on the 5th-generation tensor cores.
//
// Query rows are packed: sequence s owns rows [q_start[s], q_start[s+1]),
// which are its last q_len positions ctx - q_len .. ctx - 1; the row at
// position p attends the sequence's positions 0..p, read through its block
// table from the paged K/V pool (the causal / varlen masks of
// infrared/model/inputs.py:38-94 applied to infrared's paged read).
//
// One CTA = 128 query rows of one sequence for one query head (grid:
// q tiles x heads). Eleven warps:
//   warps 8, 9  producers: TMA copies of the Q tile (once) and of each
//               128-key K tile (warp 8) and V tile (warp 9), one box per
//               block and 64-column half, into rings of NS stages; the
//               block-table lookups are spread over the lanes and done one
//               tile ahead;
//   warp 10     MMA issuer (one thread): S = Q.K^T (M=128, N=128 keys,
//               K=D) into one of two TMEM buffers, and O += P.V (M=128,
//               N=D, K=128 keys) into the TMEM accumulator, tcgen05.mma
//               kind::f16 with operands in 128-byte-swizzled shared memory;
//               tcgen05.commit releases stages and signals the softmax;
//   warps 0-7   softmax: two threads per query row r (= TMEM lane r; warps
//               w and w + 4 share rows 32 (w % 4) ..), each takes 64 of the
//               tile's 128 keys: one 64-column TMEM load of its scores,
//               masked max (combined with the partner's through shared
//               memory), exp2 probabilities written as 16-bit P into one of
//               two shared-memory buffers (the A operand of the P.V MMA) and
//               their running sum. P is taken relative to a reference max
//               that moves only when the row max grows by more than 2^8
//               (then the row of O in TMEM and the sum are rescaled), so
//               the accumulator is rarely touched and the P.V MMA of tile j
//               overlaps the softmax of tile j + 1.
// Every wait is bounded (2 s); on a timeout the CTA flags IR_DEVERR_TIMEOUT,
// lets its copies and MMAs drain (bounded), frees its tensor memory and ends.
#include "tcgen05.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kRows = 128;     // query rows per CTA (MMA M)
constexpr int kKeys = 128;     // keys per K/V tile
constexpr int kThreads = 352;  // warps 0-7 softmax, 8-9 producers, 10 MMA
constexpr int kSoftmax = 256;  // softmax threads: 2 per query row (one per 64-key half)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;  // S buffers at columns 0 and 128, O at 256
constexpr float kRescaleLog2 = 8.f;  // move the reference max when it grows by > 2^8


template <int D>
struct PLayout {
  static constexpr int kHalves = D / 64;
  static constexpr int kHalf = kRows * 128;              // one 64-column half of a tile
  static constexpr int kQ = kHalves * kHalf;             // Q tile
  static constexpr int kSide = kHalves * kKeys * 128;    // one K or V tile
  static constexpr int NS = D == 128 ? 2 : 4;            // stages per ring
  static constexpr int kP = 2 * kHalf;                   // P: 2 halves x 128 rows x 128 B
  static constexpr int off_q = 0;
  static constexpr int off_k = kQ;
  static constexpr int off_v = off_k + NS * kSide;
  static constexpr int off_p = off_v + NS * kSide;       // two P buffers
  static constexpr int off_bar = off_p + 2 * kP;
  // q_full, q_empty, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS], s_full[2],
  // s_free[2], p_full[2], p_done[2], o_free, drain
  static constexpr int kBars = 2 + 4 * NS + 10;
  static constexpr int off_misc = off_bar + kBars * 8;
  static constexpr int off_red = off_misc + 64;         // [2 halves][128 rows] fp32 exchange
  static constexpr int kBytes = off_red + 2 * kRows * 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1 KB alignment
};

// CTA blockIdx.x -> (sequence, q tile of that sequence) by a warp-wide scan of
// tiles per sequence; seq = -1 when the index is past the last tile.
__device__ __forceinline__ void locate_tile(const PrefillArgs& a, int t, int lane, int* seq,
                                            int* tile) {
  int acc = 0;
  for (int base = 0; base < a.S; base += 32) {
    const int sq = base + lane;
    int nt = 0;
    if (sq < a.S) nt = (a.q_start[sq + 1] - a.q_start[sq] + kRows - 1) / kRows;
    if (nt < 0) nt = 0;
    int incl = nt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int excl = incl - nt;
    const bool hit = sq < a.S && t >= acc + excl && t < acc + incl;
    const unsigned bal = __ballot_sync(0xffffffffu, hit);
    if (bal) {
      const int src = __ffs(bal) - 1;
      *seq = base + src;
      *tile = t - acc - __shfl_sync(0xffffffffu, excl, src);
      return;
    }
    acc += __shfl_sync(0xffffffffu, incl, 31);
  }
  *seq = -1;
  *tile = 0;
}

// One work item: 128 query rows of one sequence for one query head.
struct Item {
  int s;      // sequence; -1: past the last item; -2: invalid metadata (skipped)
  int h, kvh;
  int r0;     // first packed query row
  int nrows;  // rows of the tile inside the sequence
  int pos0;   // position of row 0
  int n_kv;   // 128-key tiles it attends
  int ctx;
};

// Item `it` of the list (q tile major, head minor; the q tiles of a sequence
// from the last, longest one down). Warp-collective: every lane gets the same.
__device__ __forceinline__ Item item_of(const PrefillArgs& a, int it, int lane) {
  Item x;
  x.h = it % a.H;
  x.kvh = x.h / a.n_rep;
  int sq, t;
  locate_tile(a, it / a.H, lane, &sq, &t);
  x.s = sq;
  if (sq < 0) return x;
  const int qs = a.q_start[sq];
  const int ql = a.q_start[sq + 1] - qs;
  const int qt = (ql + kRows - 1) / kRows - 1 - t;
  const int ctx = a.context_lens[sq];
  if (ctx < ql || ctx > a.max_blocks * a.bs) {
    x.s = -2;
    return x;
  }
  x.r0 = qs + qt * kRows;
  x.nrows = min(kRows, ql - qt * kRows);
  x.pos0 = ctx - ql + qt * kRows;
  x.n_kv = (x.pos0 + x.nrows - 1) / kKeys + 1;
  x.ctx = ctx;
  return x;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const PrefillArgs a,
                      const int n_items) {
  using L = PLayout<D>;
  constexpr int NS = L::NS;
  constexpr bool kBf16 = DT<T>::code == IR_DTYPE_BF16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* q_empty = q_full + 1;   // the last Q.K^T of the item has completed
  uint64_t* k_full = q_empty + 1;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;  // [2] S buffer b holds tile g (g % 2 == b)
  uint64_t* s_free = s_full + 2;    // [2] the softmax has read S buffer b
  uint64_t* p_full = s_free + 2;    // [2] P buffer b written (and O rescaled)
  uint64_t* p_done = p_full + 2;    // [2] the P.V MMA reading P buffer b completed
  uint64_t* o_free = p_done + 2;    // the softmax has read the item's O
  uint64_t* drain = o_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_misc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 32) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kSoftmax);
      mbar_init(&p_full[i], kSoftmax);
      mbar_init(&p_done[i], 1);
    }
    mbar_init(o_free, kSoftmax);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    prefetch_tensormap(&tmq);
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  if (warp == 0) tc::alloc(tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Every role walks the same items in the same order; g counts the CTA's
  // K/V tiles over all its items (ring stages and S/P buffers follow g), ii
  // its items (Q buffer and O accumulator phases follow ii).

  if (warp == 8 || warp == 9) {
    // ---------------------------------------------------------- producers
    // Warp 8 loads Q and fills the K ring, warp 9 the V ring, so K tiles run
    // ahead of the V waits. Lane i < nbox resolves box i of a tile
    // (block-table lookup) one tile ahead and issues that box's copies.
    const bool is_k = warp == 8;
    uint64_t* full = is_k ? k_full : v_full;
    uint64_t* empty = is_k ? k_empty : v_empty;
    const CUtensorMap* tm = is_k ? &tmk : &tmv;
    uint8_t* ring = smem + (is_k ? L::off_k : L::off_v);
    const int R = a.bs < kKeys ? a.bs : kKeys;  // rows per box
    const int nbox = kKeys / R;                 // <= 16
    const int oob = static_cast<int>(a.num_slots);  // read as zeros by the copy
    bool ok = true;
    int g = 0, ii = 0;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const Item x = item_of(a, it, lane);
      if (x.s == -1) break;
      if (x.s < 0) continue;
      // Q of this item, once the previous item's last Q.K^T has completed
      // (issued right after the item's first K tile, which need not wait)
      auto load_q = [&]() -> bool {
        int w = 1;
        if (lane == 0) w = mbar_wait_bounded(q_empty, (ii & 1) ^ 1) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, w, 0)) return false;
        if (lane == 0) {
          mbar_arrive_expect_tx(q_full, L::kQ);
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
            tma_load_3d(smem + L::off_q + hf * L::kHalf, &tmq, q_full, 64 * hf, x.h, x.r0);
        }
        return true;
      };
      const int32_t* btr = a.block_tables + static_cast<int64_t>(x.s) * a.bt_stride;
      auto row_of = [&](int j) {
        if (lane >= nbox || j >= x.n_kv) return oob;
        const int key0 = j * kKeys + lane * R;
        if (key0 >= x.ctx) return oob;
        const int id = btr[key0 / a.bs];
        if (id < 0 || id >= a.num_blocks) {
          set_err(a.err, IR_DEVERR_BLOCK_ID);
          return oob;
        }
        return id * a.bs + key0 % a.bs;
      };
      int row_cur = row_of(0);
      for (int j = 0; j < x.n_kv; ++j, ++g) {
        const int row_next = row_of(j + 1);
        const int st = g % NS;
        int w = 1;
        if (lane == 0) w = mbar_wait_bounded(&empty[st], ((g / NS) & 1) ^ 1) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, w, 0)) {
          ok = false;
          break;
        }
        // lane i issues the copies of box i (the expected bytes are posted first)
        if (lane == 0) mbar_arrive_expect_tx(&full[st], L::kSide);
        __syncwarp();
        if (lane < nbox) {
          uint8_t* dst = ring + st * L::kSide + lane * R * 128;
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
            tma_load_3d(dst + hf * (kKeys * 128), tm, &full[st], 64 * hf, x.kvh, row_cur);
        }
        row_cur = row_next;
        if (is_k && j == 0 && !load_q()) {
          ok = false;
          ++g;
          break;
        }
      }
      ++ii;
    }
    if (lane == 0) {
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // no copy may still be writing when the CTA ends
      if (is_k && ii > 0) mbar_wait_bounded(q_full, (ii - 1) & 1);
      for (int j = g > NS ? g - NS : 0; j < g; ++j) mbar_wait_bounded(&full[j % NS], (j / NS) & 1);
    }
  } else if (warp == 10) {
    // ---------------------------------------------------------- MMA issuer
    const uint32_t qb = smem_u32(smem + L::off_q);
    const uint32_t pb = smem_u32(smem + L::off_p);
    constexpr uint32_t kIdS = tc::idesc_f16(kRows, kKeys, kBf16, false);
    constexpr uint32_t kIdO = tc::idesc_f16(kRows, D, kBf16, true);
    bool ok = true;
    int g = 0, ii = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item x = item_of(a, it, lane);
      if (x.s == -1) break;
      if (x.s < 0) continue;
      if (lane == 0) {
        auto issue_qk = [&](int gg, int j) -> bool {
          const int st = gg % NS, sb = gg & 1;
          if (!mbar_wait_bounded(&k_full[st], (gg / NS) & 1)) return false;
          if (!mbar_wait_bounded(&s_free[sb], ((gg >> 1) & 1) ^ 1)) return false;
          tc::fence_after_sync();
          const uint32_t kb = smem_u32(smem + L::off_k + st * L::kSide);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t qo = (k >> 2) * L::kHalf + (k & 3) * 32;
            const uint32_t ko = (k >> 2) * (kKeys * 128) + (k & 3) * 32;
            tc::mma_f16_ss(tmem + sb * kKeys, tc::sw128_desc(qb + qo, 16, 1024),
                           tc::sw128_desc(kb + ko, 16, 1024), kIdS, k > 0);
          }
          tc::commit(&s_full[sb]);
          tc::commit(&k_empty[st]);
          if (j == x.n_kv - 1) tc::commit(q_empty);  // the item's Q is no longer read
          return true;
        };
        auto issue_pv = [&](int gg, int j) -> bool {
          const int st = gg % NS, b = gg & 1;
          // the previous item's O has been read before this item's first P.V
          if (j == 0 && !mbar_wait_bounded(o_free, (ii & 1) ^ 1)) return false;
          if (!mbar_wait_bounded(&v_full[st], (gg / NS) & 1)) return false;
          if (!mbar_wait_bounded(&p_full[b], (gg >> 1) & 1)) return false;
          tc::fence_after_sync();
          const uint32_t vb = smem_u32(smem + L::off_v + st * L::kSide);
          const uint32_t pbb = pb + b * L::kP;
#pragma unroll
          for (int k = 0; k < kKeys / 16; ++k) {
            const uint32_t po = (k >> 2) * L::kHalf + (k & 3) * 32;
            tc::mma_f16_ss(tmem + kColO, tc::sw128_desc(pbb + po, 16, 1024),
                           tc::sw128_desc(vb + k * 2048, kKeys * 128, 1024), kIdO,
                           j > 0 || k > 0);
          }
          tc::commit(&p_done[b]);
          tc::commit(&v_empty[st]);
          return true;
        };
        ok = mbar_wait_bounded(q_full, ii & 1);
        if (ok) ok = issue_qk(g, 0);
        for (int j = 0; j < x.n_kv && ok; ++j) {
          if (j + 1 < x.n_kv) ok = issue_qk(g + j + 1, j + 1);
          if (ok) ok = issue_pv(g + j, j);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
        ok = false;
        break;
      }
      g += x.n_kv;
      ++ii;
    }
    if (lane == 0) {
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // every MMA issued has completed before the tensor memory is freed
      tc::commit(drain);
      mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int r = threadIdx.x & (kRows - 1);  // query row = TMEM lane
    const int kh = threadIdx.x >> 7;          // which 64 keys of each tile
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float* red = reinterpret_cast<float*>(smem + L::off_red);  // [2][128]
    // The two warps of a row group meet at named barrier 1 + warp % 4 (64
    // threads). They leave the loops together, right after such a meeting
    // whose AND of "all waits succeeded" is false, so neither can wait at a
    // barrier the other will not reach.
    const uint32_t pair_bar = 1 + (warp & 3);
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory"); };
    auto pair_and = [&](bool v) {
      uint32_t o;
      asm volatile(
          "{\n\t.reg .pred pi, po;\n\t"
          "setp.ne.u32 pi, %1, 0;\n\t"
          "bar.red.and.pred po, %2, 64, pi;\n\t"
          "selp.u32 %0, 1, 0, po;\n\t}"
          : "=r"(o)
          : "r"(v ? 1u : 0u), "r"(pair_bar)
          : "memory");
      return o != 0;
    };
    constexpr int kDh = D / 2;  // O columns this thread rescales / writes
    // tcgen05.ld / st are warp-collective: every wait result is made warp-uniform
    auto wait_all = [&](uint64_t* bar, uint32_t par) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, par));
    };
    bool ok = true;
    int g = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item x = item_of(a, it, lane);
      if (x.s == -1) break;
      if (x.s < 0) {
        if (threadIdx.x == 0) set_err(a.err, IR_DEVERR_CONTEXT_LEN);
        continue;
      }
      const int pos = x.pos0 + r;
      const int lim = min(pos, x.ctx - 1);  // last key this row may attend
      float m_ref = -INFINITY;  // reference max of the P values (log2 units)
      float l = 0.f;            // this half's share of the row sum
      for (int j = 0; j < x.n_kv; ++j) {
        const int gg = g + j;
        const int b = gg & 1;
        const int kbase = j * kKeys + kh * 64;
        float v[64];
        if (wait_all(&s_full[b], (gg >> 1) & 1)) {
          tc::fence_after_sync();
          tc::ld64(lane_addr + b * kKeys + kh * 64, v);
          tc::fence_before_sync();
          mbar_arrive(&s_free[b]);
        } else {
          ok = false;
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] = -INFINITY;
        }
        // keys past this row's limit exist only in the diagonal tiles: -inf there
        if (kbase + 63 > lim) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (kbase + i > lim) v[i] = -INFINITY;
        }
        float mx;
        {
          // four independent chains: v[0..3], then v[4..59] eight at a time, then v[60..63]
          float t4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
          for (int i = 4; i < 60; i += 8) {
#pragma unroll
            for (int k = 0; k < 4; ++k) t4[k] = max3(t4[k], v[i + 2 * k], v[i + 2 * k + 1]);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) t4[k] = fmaxf(t4[k], v[60 + k]);
          mx = max3(fmaxf(t4[0], t4[1]), t4[2], t4[3]);
        }
        // the row max over both halves (the partner thread holds the other 64 keys)
        red[kh * kRows + r] = mx;
        if (!pair_and(ok)) {
          ok = false;
          break;
        }
        mx = fmaxf(mx, red[(kh ^ 1) * kRows + r]) * a.scale_log2;
        pair_sync();  // both read before the next tile's write
        // move the reference max only when it has grown by more than 2^8
        const bool move = mx > m_ref + kRescaleLog2;
        const float m_new = move ? mx : m_ref;
        const float factor = ex2(m_ref - m_new);  // 0 on the first tile, 1 if not moved
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        // P buffer b is free once the P.V MMA of tile gg - 2 has completed
        if (gg >= 2 && !wait_all(&p_done[b], ((gg - 2) >> 1) & 1)) ok = false;
        // this half's keys are the 64-column half kh of the P tile
        uint8_t* prow =
            smem + L::off_p + b * L::kP + kh * L::kHalf + (r >> 3) * 1024 + (r & 7) * 128;
        // x = s * scale_log2 - m and the running sums, two keys per instruction
        const unsigned long long sc2 = f2pack(a.scale_log2, a.scale_log2);
        const unsigned long long nm2 = f2pack(-m_use, -m_use);
        unsigned long long s2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16-byte chunks of 8 keys
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const float2 xx = f2unpack(fma2(f2pack(v[c * 8 + i], v[c * 8 + i + 1]), sc2, nm2));
            const float p0 = ex2(xx.x);
            const float p1 = ex2(xx.y);
            s2[i >> 1] = add2(s2[i >> 1], f2pack(p0, p1));
            pk[i >> 1] = pack2<T>(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) * 16)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        // rows whose reference moved: O *= factor (after the P.V of tile gg - 1,
        // of this item); this thread rescales its half of the columns
        bool rescale = j > 0 && __any_sync(0xffffffffu, move);
        if (rescale && !wait_all(&p_done[(gg - 1) & 1], ((gg - 1) >> 1) & 1)) {
          ok = false;
          rescale = false;
        }
        if (rescale) {
          tc::fence_after_sync();
          const float f = move ? factor : 1.f;
#pragma unroll
          for (int c = 0; c < kDh / 32; ++c) {
            float o[32];
            const uint32_t col = kColO + kh * kDh + c * 32;
            tc::ld32(lane_addr + col, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= f;
            tc::st32(lane_addr + col, o);
          }
        }
        if (j == x.n_kv - 1 && j * kKeys + r >= x.ctx && kh < L::kHalves) {
          // key row r of the last tile lies past the context: zero its V row
          // (this thread: 64-column half kh) so that 0 * (stale pool bits)
          // cannot reach the output
          if (mbar_wait_bounded(&v_full[gg % NS], (gg / NS) & 1)) {
            uint8_t* vrow = smem + L::off_v + (gg % NS) * L::kSide + kh * (kKeys * 128) +
                            (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
            for (int k = 0; k < 8; ++k)
              *reinterpret_cast<uint4*>(vrow + k * 16) = make_uint4(0, 0, 0, 0);
          } else {
            ok = false;
          }
        }
        fence_proxy_async_shared();
        tc::fence_before_sync();
        mbar_arrive(&p_full[b]);
        const float2 u0 = f2unpack(add2(s2[0], s2[1]));
        const float2 u1 = f2unpack(add2(s2[2], s2[3]));
        l = fmaf(l, factor, (u0.x + u0.y) + (u1.x + u1.y));
        m_ref = m_new;
        // a failed wait in this tile is acted on at the next meeting
      }
      // the row sum over both halves; the pair agrees whether to go on
      red[kh * kRows + r] = l;
      const bool pok = pair_and(ok);
      const float l_row = l + red[(kh ^ 1) * kRows + r];
      pair_sync();  // both read before the next item's first write
      if (!pok) {
        ok = false;
        break;
      }
      const int gl = g + x.n_kv - 1;
      if (wait_all(&p_done[gl & 1], (gl >> 1) & 1)) {
        tc::fence_after_sync();
        const float inv = 1.f / l_row;
        T* dst = reinterpret_cast<T*>(a.out) +
                 static_cast<int64_t>(x.r0 + r) * a.out_stride +
                 static_cast<int64_t>(x.h) * D + kh * kDh;
#pragma unroll
        for (int c = 0; c < kDh / 32; ++c) {
          float o[32];
          tc::ld32(lane_addr + kColO + kh * kDh + c * 32, o);  // whole warp (collective)
          if (r < x.nrows) {
#pragma unroll
            for (int d = 0; d < 32; d += 8) {
              uint4 w;
              w.x = pack2<T>(o[d] * inv, o[d + 1] * inv);
              w.y = pack2<T>(o[d + 2] * inv, o[d + 3] * inv);
              w.z = pack2<T>(o[d + 4] * inv, o[d + 5] * inv);
              w.w = pack2<T>(o[d + 6] * inv, o[d + 7] * inv);
              *reinterpret_cast<uint4*>(dst + c * 32 + d) = w;
            }
          }
        }
        tc::fence_before_sync();
      } else {
        ok = false;
      }
      mbar_arrive(o_free);  // the next item's first P.V may overwrite O
      g += x.n_kv;
    }
    if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
    tc::fence_before_sync();
  }
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::dealloc(tmem, kTmemCols);
  }
}

template <typename T, int D>
int launch_t(const CUtensorMap& tmq, const CUtensorMap& tmk, const CUtensorMap& tmv,
             const PrefillArgs& a, int n_items, int ctas, cudaStream_t stream) {
  using L = PLayout<D>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = prefill_tc_kernel<T, D>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return static_cast<int>(e);
  kern<<<ctas, kThreads, L::kAlloc, stream>>>(tmq, tmk, tmv, a, n_items);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

int launch_prefill_tc(const CUtensorMap& tmq, const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const PrefillArgs& a, int dtype, int sm_count, cudaStream_t stream) {
  // items: an upper bound of the q tiles (every sequence adds at most one
  // partial tile) times the heads; one persistent CTA per SM walks them
  const int64_t tiles = (a.total_q + kRows - 1) / kRows + a.S;
  const int64_t items = tiles * a.H;
  if (items == 0) return 0;
  if (items > INT32_MAX) return static_cast<int>(cudaErrorInvalidValue);
  const int ctas = static_cast<int>(items < sm_count ? items : sm_count);
  const int n = static_cast<int>(items);
  if (dtype == IR_DTYPE_BF16)
    return a.D == 128 ? launch_t<__nv_bfloat16, 128>(tmq, tmk, tmv, a, n, ctas, stream)
                      : launch_t<__nv_bfloat16, 64>(tmq, tmk, tmv, a, n, ctas, stream);
  return a.D == 128 ? launch_t<__half, 128>(tmq, tmk, tmv, a, n, ctas, stream)
                    : launch_t<__half, 64>(tmq, tmk, tmv, a, n, ctas, stream);
}

}  // namespace irb
