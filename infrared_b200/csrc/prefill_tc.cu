// Paged prefill / mixed-varlen attention on the 5th-generation tensor cores.
//
// Query rows are packed: sequence s owns rows [q_start[s], q_start[s+1]),
// which are its last q_len positions ctx - q_len .. ctx - 1; the row at
// position p attends the sequence's positions 0..p, read through its block
// table from the paged K/V pool (the causal / varlen masks of
// infrared/model/inputs.py:38-94 applied to infrared's paged read).
//
// Work item = 128 query rows of one sequence for one query head; one
// persistent CTA per SM walks the items, longest first. Twelve warps:
//   warps 8, 9  producers: TMA copies of the Q tile (once) and of each
//               128-key K tile (warp 8) and V tile (warp 9), one box per
//               block and 64-column half, into rings of NS stages; the
//               block-table lookups are spread over the lanes and done one
//               tile ahead;
//   warps 10, 11 MMA issuers (one thread each, so that the tensor pipe
//               overlaps the two streams): warp 10 issues S = Q.K^T (M=128,
//               N=128 keys, K=D) into one of three TMEM buffers, up to two
//               tiles ahead of the softmax, with Q and K from
//               128-byte-swizzled shared memory; warp 11 issues
//               O += P.V (M=128, N=D, K=128 keys) into the TMEM accumulator
//               with P read from tensor memory (the A operand) and V from
//               shared memory, tcgen05.mma kind::f16; tcgen05.commit
//               releases stages and buffers and signals the softmax;
//   warps 0-7   softmax, two warpgroups taking alternate K/V tiles: thread r
//               of a warpgroup owns query row r (= TMEM lane r) and all 128
//               keys of its tiles: TMEM loads of its scores, masked max,
//               exp2 probabilities and their running sum; P goes back into
//               the same S buffer as 16-bit pairs (columns 64..127), so no
//               P passes through shared memory, whose bandwidth the MMAs
//               need. P is taken relative to a reference max that moves only
//               when the row max grows by more than 2^8 (then the row of O
//               in TMEM is rescaled); the reference is handed from tile to
//               tile through shared memory, so the two warps sharing a
//               scheduler work on different tiles at once.
//
// Pair form (PAIR, D = 128): the two CTAs of a cluster (ranks 0 and 1, one SM
// each) share 256-row work items; rank c owns rows 128c..128c+127 (its TMEM
// lanes and its softmax warps) and the pair's tensor cores run one
// tcgen05.mma.cta_group::2 of M = 256 per step, issued by rank 0. Each CTA
// stages half of every K tile (64 keys, all of D) and half of every V tile
// (all 128 keys, its 64 columns of D): the MMA reads the B operand's halves
// from both SMs, so each SM moves half the K/V bytes through its shared
// memory and Q.K^T reads 6 KB instead of 8 KB of it per 16-element step.
// Barriers counting both CTAs (stage full, Q full, P full, O free) live in
// rank 0: rank 1's copies complete on them across the pair and its softmax
// threads arrive on them remotely; rank 0's commits signal both CTAs' copies
// of the per-CTA barriers (stage empty, S full, P.V done) at once.
//
// Every wait is bounded (2 s); on a timeout the CTA flags IR_DEVERR_TIMEOUT,
// lets its copies and MMAs drain (bounded), frees its tensor memory and ends.
#include "tcgen05.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kRows = 128;     // query rows per CTA (MMA M)
constexpr int kKeys = 128;     // keys per K/V tile
// warps 0-7 softmax (two warpgroups), 8-9 producers, 10 Q.K^T issuer, 11 P.V issuer
constexpr int kThreads = 384;
constexpr int kWgThreads = 128;  // one softmax warpgroup: one thread per query row
constexpr uint32_t kTmemCols = 512;
constexpr int kSBuf = 3;  // S buffers: Q.K^T runs two tiles ahead of the softmax
constexpr uint32_t kColO = kSBuf * kKeys;  // S buffers at columns 0, 128, 256; O at 384
constexpr int kPairStages = 2;  // ring stages of the pair form (16 KB per side each)
constexpr float kRescaleLog2 = 8.f;  // move the reference max when it grows by > 2^8


template <int D, bool PAIR>
struct PLayout {
  static constexpr int kHalves = D / 64;
  static constexpr int kHalf = kRows * 128;              // one 64-column half of the Q tile
  static constexpr int kQ = kHalves * kHalf;             // Q tile (this CTA's rows)
  // keys of a K tile staged here (a pair splits them) and one 64-column half of them
  static constexpr int kKRows = PAIR ? kKeys / 2 : kKeys;
  static constexpr int kKHalf = kKRows * 128;
  static constexpr int kKSide = kHalves * kKHalf;
  // 64-column halves of a V tile staged here (a pair splits the columns)
  static constexpr int kVHalves = PAIR ? 1 : kHalves;
  static constexpr int kVSide = kVHalves * kKeys * 128;
  static constexpr int NS = PAIR ? kPairStages : (D == 128 ? 2 : 4);  // stages per ring
  static constexpr int off_q = 0;
  static constexpr int off_k = kQ;
  static constexpr int off_v = off_k + NS * kKSide;
  static constexpr int off_bar = off_v + NS * kVSide;
  // q_full, q_empty, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS], s_full[kSBuf],
  // s_free[kSBuf], p_full[2], p_done[2], o_free, drain, ref_full[2], l_ready, v_last
  static constexpr int kBars = 2 + 4 * NS + 2 * kSBuf + 10;
  static constexpr int off_misc = off_bar + kBars * 8;
  // reference max per row after tile g, [g & 1][128 rows], then the row sums one
  // softmax warpgroup hands to the other at the end of an item [128 rows]
  static constexpr int off_ref = off_misc + 64;
  static constexpr int kBytes = off_ref + 3 * kRows * 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1 KB alignment
};

// Tile index t -> (sequence, q tile of that sequence) by a warp-wide scan of
// TR-row tiles per sequence; seq = -1 when the index is past the last tile.
template <int TR>
__device__ __forceinline__ void locate_tile(const PrefillArgs& a, int t, int lane, int* seq,
                                            int* tile) {
  int acc = 0;
  for (int base = 0; base < a.S; base += 32) {
    const int sq = base + lane;
    int nt = 0;
    if (sq < a.S) nt = (a.q_start[sq + 1] - a.q_start[sq] + TR - 1) / TR;
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

// One work item: TR (128, or 256 for a CTA pair) query rows of one sequence
// for one query head.
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
template <int TR = kRows>
__device__ __forceinline__ Item item_of(const PrefillArgs& a, int it, int lane) {
  Item x;
  x.h = it % a.H;
  x.kvh = x.h / a.n_rep;
  int sq, t;
  locate_tile<TR>(a, it / a.H, lane, &sq, &t);
  x.s = sq;
  if (sq < 0) return x;
  const int qs = a.q_start[sq];
  const int ql = a.q_start[sq + 1] - qs;
  const int qt = (ql + TR - 1) / TR - 1 - t;
  const int ctx = a.context_lens[sq];
  if (ctx < ql || ctx > a.max_blocks * a.bs) {
    x.s = -2;
    return x;
  }
  x.r0 = qs + qt * TR;
  x.nrows = min(TR, ql - qt * TR);
  x.pos0 = ctx - ql + qt * TR;
  x.n_kv = (x.pos0 + x.nrows - 1) / kKeys + 1;
  x.ctx = ctx;
  return x;
}


template <typename T, int D, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const PrefillArgs a,
                      const int n_items) {
  static_assert(!PAIR || D == 128, "the pair form takes D = 128");
  using L = PLayout<D, PAIR>;
  constexpr int NS = L::NS;
  constexpr int TR = PAIR ? 2 * kRows : kRows;  // query rows of a work item
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
  uint64_t* s_full = v_empty + NS;    // [kSBuf] S buffer b holds tile g (g % kSBuf == b)
  uint64_t* s_free = s_full + kSBuf;  // [kSBuf] the P.V reading P from S buffer b completed
  uint64_t* p_full = s_free + kSBuf;  // [2] P of tile g (g & 1 == b) written, O rescaled
  uint64_t* p_done = p_full + 2;      // [2] the P.V MMA of tile g (g & 1 == b) completed
  uint64_t* o_free = p_done + 2;      // the softmax has read the item's O
  uint64_t* drain = o_free + 1;
  uint64_t* ref_full = drain + 1;     // [2] the reference max after tile g is in sref[g & 1]
  uint64_t* l_ready = ref_full + 2;   // the other warpgroup's row sums are in lsum
  uint64_t* v_last = l_ready + 1;     // pair: this CTA's V half of an item's last tile landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_misc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool lead = rank == 0;  // issues the MMAs (always, without a pair)
  // the items are dealt over CTAs, or over pairs
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  constexpr uint32_t kBoth = PAIR ? 2u : 1u;  // CTAs whose stage bytes rank 0 counts
  // Fewer commits per tile: with a 2-stage ring, a K stage is free once the
  // Q.K^T of the tile two back completed (S full) and a V stage once its P.V
  // did (P.V done), so those barriers stand in for K empty and V empty. No
  // phase can alias: the next phase of each needs a tile that the waiting
  // producer has not loaded yet.
  constexpr bool kLean = NS == 2;
  // arrivals on P full / O free: every softmax thread of the CTA (of both CTAs
  // of a pair)
  constexpr uint32_t kSoftArrivals = kBoth * kWgThreads;

  if (threadIdx.x == 32) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < kSBuf; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], kSoftArrivals);
      mbar_init(&p_done[i], 1);
      mbar_init(&ref_full[i], kWgThreads);
    }
    mbar_init(o_free, kSoftArrivals);
    mbar_init(drain, 2);  // one commit from each MMA issuer
    mbar_init(l_ready, kWgThreads);
    mbar_init(v_last, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    prefetch_tensormap(&tmq);
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  // both CTAs of a pair have initialised their barriers before either signals
  // the other's, and both are running before the pair allocates
  if constexpr (PAIR) cluster_sync();
  if (warp == 0) {
    if constexpr (PAIR)
      tc::alloc2(tmem_slot, kTmemCols);  // warp 0 of both CTAs: the same columns in each
    else
      tc::alloc(tmem_slot, kTmemCols);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Every role walks the same items in the same order; g counts the CTA's
  // K/V tiles over all its items (ring stages and S buffers follow g), ii
  // its items (Q buffer, O accumulator and v_last phases follow ii).

  if (warp == 8 || warp == 9) {
    // ---------------------------------------------------------- producers
    // Warp 8 loads Q and fills the K ring, warp 9 the V ring, so K tiles run
    // ahead of the V waits. Lane i < nbox resolves box i of a tile
    // (block-table lookup) one tile ahead and issues that box's copies.
    // In a pair, rank 0 posts the bytes of both CTAs on its full barriers
    // and both CTAs' copies complete there.
    const bool is_k = warp == 8;
    uint64_t* full = is_k ? k_full : v_full;
    uint64_t* empty = is_k ? k_empty : v_empty;
    const CUtensorMap* tm = is_k ? &tmk : &tmv;
    uint8_t* ring = smem + (is_k ? L::off_k : L::off_v);
    const int side = is_k ? L::kKSide : L::kVSide;
    const int span = is_k ? L::kKRows : kKeys;  // keys of a tile staged here
    const int first = is_k ? static_cast<int>(rank) * L::kKRows : 0;  // the first of them
    // 64-column halves staged here: all for K; for V one per CTA of a pair
    const int half0 = is_k ? 0 : static_cast<int>(rank);  // the first of them
    const int halfb = span * 128;                        // bytes of one staged half
    const int R = a.bs < span ? a.bs : span;             // rows per box
    const int nbox = span / R;                           // <= 16
    const int oob = static_cast<int>(a.num_slots);  // read as zeros by the copy
    bool ok = true;
    int g = 0, ii = 0;
    int g_prev = -1;  // the previous item's last tile
    for (int it = unit; it < n_items && ok; it += units) {
      const Item x = item_of<TR>(a, it, lane);
      if (x.s == -1) break;
      if (x.s < 0) continue;
      // Q of this item, once the previous item's last Q.K^T has completed
      // (issued right after the item's first K tile, which need not wait)
      auto load_q = [&]() -> bool {
        int w = 1;
        if (lane == 0) w = mbar_wait_bounded(q_empty, (ii & 1) ^ 1) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, w, 0)) return false;
        if (lane == 0) {
          const int qrow = x.r0 + static_cast<int>(rank) * kRows;
          if constexpr (PAIR) {
            if (lead) mbar_arrive_expect_tx(q_full, 2 * L::kQ);
            const uint32_t cb = cluster_addr(q_full, 0);
#pragma unroll
            for (int hf = 0; hf < L::kHalves; ++hf)
              tma_load_3d_pair(smem + L::off_q + hf * L::kHalf, &tmq, cb, 64 * hf, x.h, qrow);
          } else {
            mbar_arrive_expect_tx(q_full, L::kQ);
#pragma unroll
            for (int hf = 0; hf < L::kHalves; ++hf)
              tma_load_3d(smem + L::off_q + hf * L::kHalf, &tmq, q_full, 64 * hf, x.h, qrow);
          }
        }
        return true;
      };
      const int32_t* btr = a.block_tables + static_cast<int64_t>(x.s) * a.bt_stride;
      auto row_of = [&](int j) {
        if (lane >= nbox || j >= x.n_kv) return oob;
        const int key0 = j * kKeys + first + lane * R;
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
        // a pair's V half of the item's last tile completes on this CTA's own
        // v_last, so that its softmax can zero the rows past the context
        // before the P.V reads them (rank 0's full barrier then only counts
        // the phase; P full covers the data)
        const bool last_v = PAIR && !is_k && j == x.n_kv - 1;
        int w = 1;
        if (lane == 0) {
          if (!kLean)
            w = mbar_wait_bounded(&empty[st], ((g / NS) & 1) ^ 1) ? 1 : 0;
          else if (g >= NS)
            w = (is_k ? mbar_wait_bounded(&s_full[(g - NS) % kSBuf], ((g - NS) / kSBuf) & 1)
                      : mbar_wait_bounded(&p_done[(g - NS) & 1], ((g - NS) >> 1) & 1))
                    ? 1
                    : 0;
          // v_last takes its next phase only after the P.V of the previous
          // item's last tile (whose softmax waited on the previous phase)
          // completed; a wait the ring wait above already implies is skipped
          if (w && last_v && g_prev >= 0 && g - g_prev < NS)
            w = (kLean ? mbar_wait_bounded(&p_done[g_prev & 1], (g_prev >> 1) & 1)
                       : mbar_wait_bounded(&empty[g_prev % NS], (g_prev / NS) & 1))
                    ? 1
                    : 0;
        }
        if (!__shfl_sync(0xffffffffu, w, 0)) {
          ok = false;
          break;
        }
        // lane i issues the copies of box i (the expected bytes are posted first)
        if (lane == 0) {
          if (last_v) {
            mbar_arrive_expect_tx(v_last, side);
            if (lead) mbar_arrive(&full[st]);
          } else if (lead) {
            mbar_arrive_expect_tx(&full[st], kBoth * side);
          }
        }
        __syncwarp();
        if (lane < nbox) {
          uint8_t* dst = ring + st * side + lane * R * 128;
          const uint32_t cb = PAIR ? cluster_addr(&full[st], 0) : 0u;
#pragma unroll
          for (int hf = 0; hf < (is_k ? L::kHalves : L::kVHalves); ++hf) {
            const int col = 64 * (half0 + hf);
            if (!PAIR)
              tma_load_3d(dst + hf * halfb, tm, &full[st], col, x.kvh, row_cur);
            else if (last_v)
              tma_load_3d(dst + hf * halfb, tm, v_last, col, x.kvh, row_cur);
            else
              tma_load_3d_pair(dst + hf * halfb, tm, cb, col, x.kvh, row_cur);
          }
        }
        row_cur = row_next;
        if (is_k && j == 0 && !load_q()) {
          ok = false;
          ++g;
          break;
        }
      }
      g_prev = g - 1;
      ++ii;
    }
    if (lane == 0) {
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // no copy may still be writing when the CTA ends: rank 0's full
      // barriers count both CTAs' copies (a pair leaves together)
      if (lead) {
        if (is_k && ii > 0) mbar_wait_bounded(q_full, (ii - 1) & 1);
        for (int j = g > NS ? g - NS : 0; j < g; ++j)
          mbar_wait_bounded(&full[j % NS], (j / NS) & 1);
      }
      if (PAIR && !is_k && ii > 0) mbar_wait_bounded(v_last, (ii - 1) & 1);
    }
  } else if (warp == 10 || warp == 11) {
    // ---------------------------------------------------------- MMA issuers
    // Warp 10 issues the Q.K^T MMAs and warp 11 the P.V MMAs (one thread
    // each): MMAs issued from two threads overlap in the tensor pipe, where
    // one thread's stream runs them one after the other (a 128 x 128 x 16
    // Q.K^T + P.V pair: ~118 cycles from two threads, ~187 from one). Rank 0
    // of a pair issues for both CTAs; rank 1's two warps idle.
    const bool is_qk = warp == 10;
    auto mma_ss = [](uint32_t d, uint64_t ad, uint64_t bd, uint32_t id, bool acc) {
      if constexpr (PAIR)
        tc::mma2_f16_ss(d, ad, bd, id, acc);
      else
        tc::mma_f16_ss(d, ad, bd, id, acc);
    };
    auto mma_ts = [](uint32_t d, uint32_t at, uint64_t bd, uint32_t id, bool acc) {
      if constexpr (PAIR)
        tc::mma2_f16_ts(d, at, bd, id, acc);
      else
        tc::mma_f16_ts(d, at, bd, id, acc);
    };
    // signal a barrier in both CTAs of a pair, or in rank 0 only
    auto commit_both = [](uint64_t* bar) {
      if constexpr (PAIR)
        tc::commit2(bar, 3);
      else
        tc::commit(bar);
    };
    auto commit_lead = [](uint64_t* bar) {
      if constexpr (PAIR)
        tc::commit2(bar, 1);
      else
        tc::commit(bar);
    };
    // P full / O free collect arrivals from both CTAs of a pair; the item's
    // last P follows shared-memory writes of the peer (zeroed V rows) released
    // at cluster scope, so that wait acquires at cluster scope
    auto wait_both = [](uint64_t* bar, uint32_t par, bool cluster_scope) {
      return PAIR && cluster_scope ? mbar_wait_bounded_cluster(bar, par)
                                   : mbar_wait_bounded(bar, par);
    };
    const uint32_t qb = smem_u32(smem + L::off_q);
    constexpr uint32_t kIdS = tc::idesc_f16(PAIR ? 2 * kRows : kRows, kKeys, kBf16, false);
    constexpr uint32_t kIdO = tc::idesc_f16(PAIR ? 2 * kRows : kRows, D, kBf16, true);
    bool ok = true;
    int g = 0, ii = 0;
    for (int it = unit; it < n_items && lead; it += units) {
      const Item x = item_of<TR>(a, it, lane);
      if (x.s == -1) break;
      if (x.s < 0) continue;
      if (lane == 0 && is_qk) {
        // S = Q.K^T of each tile into S buffer g % 3, as soon as the K tile
        // has landed and the P.V of the tile three back has read that buffer
        ok = mbar_wait_bounded(q_full, ii & 1);
        for (int j = 0; j < x.n_kv && ok; ++j) {
          const int gg = g + j, st = gg % NS, sb = gg % kSBuf;
          ok = mbar_wait_bounded(&k_full[st], (gg / NS) & 1) &&
               mbar_wait_bounded(&s_free[sb], ((gg / kSBuf) & 1) ^ 1);
          if (!ok) break;
          tc::fence_after_sync();
          const uint32_t kb = smem_u32(smem + L::off_k + st * L::kKSide);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t qo = (k >> 2) * L::kHalf + (k & 3) * 32;
            const uint32_t ko = (k >> 2) * L::kKHalf + (k & 3) * 32;
            mma_ss(tmem + sb * kKeys, tc::sw128_desc(qb + qo, 16, 1024),
                   tc::sw128_desc(kb + ko, 16, 1024), kIdS, k > 0);
          }
          commit_both(&s_full[sb]);
          if (!kLean) commit_both(&k_empty[st]);
          if (j == x.n_kv - 1) commit_both(q_empty);  // the item's Q is no longer read
        }
      } else if (lane == 0) {
        // O += P.V of each tile once its P is in tensor memory (and, at an
        // item's first tile, the previous item's O has been read)
        for (int j = 0; j < x.n_kv && ok; ++j) {
          const int gg = g + j, st = gg % NS, b = gg & 1, sb = gg % kSBuf;
          ok = (j > 0 || wait_both(o_free, (ii & 1) ^ 1, false)) &&
               wait_both(&p_full[b], (gg >> 1) & 1, j == x.n_kv - 1) &&
               mbar_wait_bounded(&v_full[st], (gg / NS) & 1);
          if (!ok) break;
          tc::fence_after_sync();
          const uint32_t vb = smem_u32(smem + L::off_v + st * L::kVSide);
          // P (16-bit, two keys per column) sits in columns 64..127 of S buffer sb
          const uint32_t pt = tmem + sb * kKeys + 64;
#pragma unroll
          for (int k = 0; k < kKeys / 16; ++k)
            mma_ts(tmem + kColO, pt + k * 8, tc::sw128_desc(vb + k * 2048, kKeys * 128, 1024),
                   kIdO, j > 0 || k > 0);
          commit_both(&p_done[b]);
          commit_lead(&s_free[sb]);  // S buffer sb (holding P) may take Q.K^T again
          if (!kLean) commit_both(&v_empty[st]);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
        ok = false;
        break;
      }
      g += x.n_kv;
      ++ii;
    }
    if (lead && lane == 0) {
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // every MMA issued has completed before the tensor memory is freed
      // (and, in a pair, before either CTA's shared memory goes away): the
      // drain barrier counts both issuers' commits
      commit_lead(drain);
      mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    // Two warpgroups take alternate K/V tiles (warpgroup g & 1 takes the
    // CTA's tile g); thread r of a warpgroup owns query row r (= TMEM lane r)
    // and all 128 keys of its tiles, so the two warps that share a scheduler
    // work on different tiles and overlap. What crosses from one tile to the
    // next is the row's reference max: tile g stores the reference its P
    // values use in sref[g & 1] and arrives on ref_full[g & 1]; tile g + 1
    // waits for it. (Slot g & 1 is written again by tile g + 2 only after
    // that tile has seen tile g + 1's reference, which tile g + 1 published
    // after reading slot g & 1.) Each warpgroup keeps its own row sums; at the
    // end of an item the other warpgroup hands its sums to the warpgroup of
    // the item's last tile through lsum / l_ready, and that one normalises
    // and writes the item's rows and releases O. In a pair, rank c's thread r
    // owns item row 128c + r, and the P full / O free arrivals go to rank 0.
    const int wg = warp >> 2;
    const int r = threadIdx.x & (kRows - 1);  // query row = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float* sref = reinterpret_cast<float*>(smem + L::off_ref);  // [2][128]
    float* lsum = sref + 2 * kRows;                              // [128]
    const int rbase = static_cast<int>(rank) * kRows;  // this CTA's first row of an item
    const uint32_t c_pfull0 = PAIR ? cluster_addr(&p_full[0], 0) : 0u;
    const uint32_t c_pfull1 = PAIR ? cluster_addr(&p_full[1], 0) : 0u;
    const uint32_t c_ofree = PAIR ? cluster_addr(o_free, 0) : 0u;
    // In a pair every softmax thread arrives on rank 0's barrier: P and O live
    // in tensor memory, ordered by tcgen05.fence::before_thread_sync, and a
    // CTA-scope release hands them over; only a tile whose V rows this
    // thread zeroed in shared memory releases at cluster scope
    auto arrive_p_full = [&](int b, bool wrote_smem) {
      if constexpr (PAIR) {
        const uint32_t cb = b ? c_pfull1 : c_pfull0;
        if (wrote_smem)
          mbar_arrive_cluster(cb);
        else
          mbar_arrive_remote(cb);
      } else {
        mbar_arrive(&p_full[b]);
      }
    };
    auto arrive_o_free = [&]() {
      if constexpr (PAIR)
        mbar_arrive_remote(c_ofree);
      else
        mbar_arrive(o_free);
    };
    bool ok = true;
    // tcgen05.ld / st are warp-collective: every wait result is warp-uniform;
    // after a failed wait the remaining waits are skipped (arrivals go on), so
    // the walk ends quickly and the other roles' bounded waits end theirs
    auto wait_all = [&](uint64_t* bar, uint32_t par) {
      if (!ok) return false;
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, par));
      return ok;
    };
    const unsigned long long sc2 = f2pack(a.scale_log2, a.scale_log2);
    // keys past this row's limit exist only in the diagonal tiles: -inf there
    auto mask = [&](float (&v)[64], int k0, int lim) {
      if (k0 + 63 > lim) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (k0 + i > lim) v[i] = -INFINITY;
      }
    };
    auto half_max = [&](const float (&v)[64]) {
      // four independent chains: v[0..3], then v[4..59] eight at a time, then v[60..63]
      float t4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
      for (int i = 4; i < 60; i += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k) t4[k] = max3(t4[k], v[i + 2 * k], v[i + 2 * k + 1]);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) t4[k] = fmaxf(t4[k], v[60 + k]);
      return max3(fmaxf(t4[0], t4[1]), t4[2], t4[3]);
    };
    // p = 2^(s * scale_log2 - m) for 64 keys, summed two at a time and
    // written as 16-bit P, two keys per column, into this row's TMEM lane at
    // column `col` (32 columns): the A operand of the P.V MMA
    auto exp_store = [&](const float (&v)[64], uint32_t col, unsigned long long nm2,
                         unsigned long long (&s2)[4]) {
      float pk[32];
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float2 xx = f2unpack(fma2(f2pack(v[i], v[i + 1]), sc2, nm2));
        const float p0 = ex2(xx.x);
        const float p1 = ex2(xx.y);
        s2[(i >> 1) & 3] = add2(s2[(i >> 1) & 3], f2pack(p0, p1));
        pk[i >> 1] = __uint_as_float(pack2<T>(p0, p1));
      }
      tc::st32(lane_addr + col, pk);  // waits for the store
    };
    int g = 0, ii = 0;
    for (int it = unit; it < n_items; it += units) {
      const Item x = item_of<TR>(a, it, lane);
      if (x.s == -1) break;
      if (x.s < 0) {
        if (threadIdx.x == 0) set_err(a.err, IR_DEVERR_CONTEXT_LEN);
        continue;
      }
      const int pos = x.pos0 + rbase + r;
      const int lim = min(pos, x.ctx - 1);  // last key this row may attend
      const int gl = g + x.n_kv - 1;        // the item's last tile
      float l = 0.f;           // this warpgroup's part of the row sum, relative to m_l
      float m_l = -INFINITY;   // the reference of this warpgroup's last tile
      for (int j = (wg - g) & 1; j < x.n_kv; j += 2) {
        const int gg = g + j;
        const int b = gg & 1;         // barrier parity slot and reference slot (== wg)
        const int sb = gg % kSBuf;    // S buffer
        const int k0 = j * kKeys;
        float v[64];
        // the row max over the tile: keys 0-63, then 64-127 (kept in registers)
        float mx = -INFINITY;
        if (wait_all(&s_full[sb], (gg / kSBuf) & 1)) {
          tc::fence_after_sync();
          tc::ld64(lane_addr + sb * kKeys, v);
          mask(v, k0, lim);
          mx = half_max(v);
          // the first half's max is taken before the second half is loaded:
          // 64 scores live at a time, not 128
          asm volatile("" ::"f"(mx));
          tc::ld64(lane_addr + sb * kKeys + 64, v);
          mask(v, k0 + 64, lim);
          mx = fmaxf(mx, half_max(v)) * a.scale_log2;
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] = -INFINITY;
        }
        // the reference of the previous tile (none at an item's first tile)
        float prev = -INFINITY;
        if (gg > 0 && wait_all(&ref_full[(gg - 1) & 1], ((gg - 1) >> 1) & 1) && j > 0)
          prev = sref[((gg - 1) & 1) * kRows + r];
        // move the reference only when the max has grown by more than 2^8
        const bool move = mx > prev + kRescaleLog2;
        const float m_new = move ? mx : prev;
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        sref[b * kRows + r] = m_use;
        mbar_arrive(&ref_full[b]);
        // P goes to columns 64..127 of S buffer sb: keys 64-127 (in registers)
        // first, into columns 96..127, whose scores are no longer needed;
        // then keys 0-63, read again from columns 0..63, into 64..95
        const uint32_t pcol = sb * kKeys + 64;
        const unsigned long long nm2 = f2pack(-m_use, -m_use);
        unsigned long long s2[4] = {0ull, 0ull, 0ull, 0ull};
        exp_store(v, pcol + 32, nm2, s2);
        asm volatile("" ::: "memory");  // keys 64-127 are stored before anything below
        // rows whose reference moved: O *= 2^(prev - m_use), after the P.V of
        // tile gg - 1 (this item's) and before this tile's
        if (j > 0 && __any_sync(0xffffffffu, move) &&
            wait_all(&p_done[(gg - 1) & 1], ((gg - 1) >> 1) & 1)) {
          tc::fence_after_sync();
          const float f = move ? ex2(prev - m_use) : 1.f;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            const uint32_t col = kColO + c * 32;
            tc::ld32(lane_addr + col, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= f;
            tc::st32(lane_addr + col, o);
          }
        }
        // keys 0-63 again (unconditionally: a skipped load would keep keys
        // 64-127 live through the pass above; after a failed wait the
        // values are unused garbage in allocated tensor memory)
        tc::ld64(lane_addr + sb * kKeys, v);
        mask(v, k0, lim);
        exp_store(v, pcol, nm2, s2);
        bool zeroed = false;
        if (j == x.n_kv - 1) {
          // key row r of the last tile past the context: zero its V row (this
          // CTA's columns) so that 0 * (stale pool bits) cannot reach the output
          const int vst = gg % NS;
          bool landed;
          if constexpr (PAIR)
            landed = wait_all(v_last, ii & 1);
          else
            landed = __any_sync(0xffffffffu, k0 + r >= x.ctx) &&
                     wait_all(&v_full[vst], (gg / NS) & 1);
          if (landed && k0 + r >= x.ctx) {
            zeroed = true;
#pragma unroll
            for (int h = 0; h < L::kVHalves; ++h) {
              uint8_t* vrow = smem + L::off_v + vst * L::kVSide + h * (kKeys * 128) +
                              (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
              for (int k = 0; k < 8; ++k)
                *reinterpret_cast<uint4*>(vrow + k * 16) = make_uint4(0, 0, 0, 0);
            }
          }
        }
        fence_proxy_async_shared();
        tc::fence_before_sync();
        arrive_p_full(b, zeroed);
        const float2 u0 = f2unpack(add2(s2[0], s2[1]));
        const float2 u1 = f2unpack(add2(s2[2], s2[3]));
        const float fl = m_l == m_use ? 1.f : ex2(m_l - m_use);  // 0 before the first tile
        l = fmaf(l, fl, (u0.x + u0.y) + (u1.x + u1.y));
        m_l = m_use;
      }
      if ((gl & 1) != wg) {
        // hand this warpgroup's sums, relative to the item's last reference,
        // to the warpgroup of the last tile
        float m_fin = m_l;
        if (wait_all(&ref_full[gl & 1], (gl >> 1) & 1)) m_fin = sref[(gl & 1) * kRows + r];
        lsum[r] = m_l == m_fin ? l : l * ex2(m_l - m_fin);
        mbar_arrive(l_ready);
      } else {
        float lo = 0.f;
        if (wait_all(l_ready, ii & 1)) lo = lsum[r];
        const float l_row = l + lo;
        if (wait_all(&p_done[gl & 1], (gl >> 1) & 1)) {
          tc::fence_after_sync();
          const float inv = 1.f / l_row;
          T* dst = reinterpret_cast<T*>(a.out) +
                   static_cast<int64_t>(x.r0 + rbase + r) * a.out_stride +
                   static_cast<int64_t>(x.h) * D;
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            float o[32];
            tc::ld32(lane_addr + kColO + c * 32, o);  // whole warp (collective)
            if (rbase + r < x.nrows) {
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
            asm volatile("" ::: "memory");  // one 32-column chunk live at a time
          }
          tc::fence_before_sync();
        }
        arrive_o_free();  // the next item's first P.V may overwrite O
      }
      g += x.n_kv;
      ++ii;
    }
    if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
    tc::fence_before_sync();
  }
  __syncthreads();
  // neither CTA of a pair leaves while its peer may still signal its
  // barriers, read its shared memory or write its tensor memory
  if constexpr (PAIR) cluster_sync();
  if (warp == 0) {
    tc::fence_after_sync();
    if constexpr (PAIR)
      tc::dealloc2(tmem, kTmemCols);
    else
      tc::dealloc(tmem, kTmemCols);
  }
}


template <typename T, int D, bool PAIR>
int launch_t(const CUtensorMap& tmq, const CUtensorMap& tmk, const CUtensorMap& tmv,
             const PrefillArgs& a, int n_items, int sm_count, cudaStream_t stream) {
  using L = PLayout<D, PAIR>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = prefill_tc_kernel<T, D, PAIR>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return static_cast<int>(e);
  if constexpr (!PAIR) {
    // one persistent CTA per SM
    const int ctas = n_items < sm_count ? n_items : sm_count;
    kern<<<ctas, kThreads, L::kAlloc, stream>>>(tmq, tmk, tmv, a, n_items);
    return static_cast<int>(cudaGetLastError());
  } else {
    // one persistent pair per pair of SMs that can hold one at a time
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kAlloc;
    cfg.stream = stream;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(sm_count & ~1));
    static int resident = 0;  // pairs the device holds at once (asked once)
    int clusters = resident;
    if (clusters <= 0) {
      if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
        (void)cudaGetLastError();
        clusters = sm_count / 2;
      } else {
        resident = clusters;
      }
    }
    const int pairs = n_items < clusters ? n_items : clusters;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    e = cudaLaunchKernelEx(&cfg, kern, tmq, tmk, tmv, a, n_items);
    return static_cast<int>(e);
  }
}

}  // namespace

int launch_prefill_tc(const CUtensorMap& tmq, const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const PrefillArgs& a, int dtype, int sm_count, bool pair,
                      cudaStream_t stream) {
  // items: an upper bound of the q tiles (every sequence adds at most one
  // partial tile) times the heads; persistent CTAs (or pairs) walk them
  const int tr = pair ? 2 * kRows : kRows;
  const int64_t tiles = (a.total_q + tr - 1) / tr + a.S;
  const int64_t items = tiles * a.H;
  if (items == 0) return 0;
  if (items > INT32_MAX) return static_cast<int>(cudaErrorInvalidValue);
  const int n = static_cast<int>(items);
  if (pair) {
    if (a.D != 128) return static_cast<int>(cudaErrorInvalidValue);
    return dtype == IR_DTYPE_BF16
               ? launch_t<__nv_bfloat16, 128, true>(tmq, tmk, tmv, a, n, sm_count, stream)
               : launch_t<__half, 128, true>(tmq, tmk, tmv, a, n, sm_count, stream);
  }
  if (dtype == IR_DTYPE_BF16)
    return a.D == 128 ? launch_t<__nv_bfloat16, 128, false>(tmq, tmk, tmv, a, n, sm_count, stream)
                      : launch_t<__nv_bfloat16, 64, false>(tmq, tmk, tmv, a, n, sm_count, stream);
  return a.D == 128 ? launch_t<__half, 128, false>(tmq, tmk, tmv, a, n, sm_count, stream)
                    : launch_t<__half, 64, false>(tmq, tmk, tmv, a, n, sm_count, stream);
}

}  // namespace irb
