// Paged decode attention for 16-bit pools: TMA-fed, warp-specialised.
//
// A CTA owns a group of HG kv heads and one share of the 16-token tiles of
// every sequence (decode_common.cuh). Warp 0 is the producer: its lanes
// resolve 32 tiles at a time (sequence walk + block-table lookup), then lane
// 0 issues, per tile, one TMA tensor copy for K and one for V that move the
// tile's rows for all HG heads at once (HG x 16 rows x D x 2 B = 16 KB for
// HG = 4, D = 128 — one contiguous piece of a block). The tensor map views a
// pool row as [head][half][64 elements] with dimensions ordered
// (element, slot, half, head), so the box lands in shared memory as one
// 2 KB region per (head, 64-column half) of 16 rows x 128 B with the 128-byte
// swizzle, which makes the ldmatrix reads below conflict free. Stages are
// guarded by full/empty mbarriers.
//
// Warps 1..HG are consumers, one per kv head; each sees every tile. For its
// head, per tile, it computes for the whole GQA group at once (padded to 8
// columns):
//   S^T[16 tok x 8 heads] = K[16 x D] . Q^T[D x 8]    (D/16 mma.m16n8k16)
//   online softmax over the 16 tokens per head (exp2 on the SFU, fp32)
//   O^T[D x 8]           += V^T[D x 16] . P^T[16 x 8]  (D/16 mma.m16n8k16)
// with P^T moved into B-operand layout by two movmatrix transposes, so each
// K/V element is read from HBM once for the whole group. The tensor-core
// instructions are the warp-level mma.sync form: the path is bound by HBM
// bandwidth, and mma.sync only removes the FMA/convert issue that would
// otherwise cap a CUDA-core GEMV at ~7 FMAs per loaded element. A warp writes
// its segment's row (or workspace piece) itself when the sequence changes;
// no cross-warp combine is needed.
//
// With the dynamic tail (DecodeArgs::dyn, decode_common.cuh) the producer
// streams its static unit, then claims dynamic units from the workspace
// counter until none is left; a unit start is a segment start, and the unit
// index travels to the consumers in the item descriptor (pieces sit in slot
// unit + b). Every CTA counts itself done at its end; the last CTA of the
// kv-head group sets the counters back to zero.
//
// With the in-kernel merge (DecodeArgs::inline_merge) a warp that writes a
// piece of a row split into at most kInlineMax pieces counts it in the row's
// counter (ws_seq); the warp that writes the last one merges the row's
// pieces in unit order right away, while the other CTAs are still
// streaming, and sets the counter back to zero; the merge kernel then skips
// those rows. The producer packs the row's piece count and this piece's
// index into the item descriptor.
#include "decode_common.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr unsigned kFull = 0xffffffffu;

struct __align__(16) ItemDesc {
  int b;
  int tok0;
  int seg;     // (unit << 1) | (segment index & 1): workspace unit, q buffer
  int packed;  // n_valid in bits 0-7, flags above
};
constexpr int kFlagValid = 1 << 8;     // copies were issued (block ids valid)
constexpr int kFlagSeqEnd = 1 << 9;    // last tile of the sequence
constexpr int kFlagWhole = 1 << 10;    // the segment is the whole sequence
constexpr int kFlagEnd = 1 << 11;      // end-of-stream marker
constexpr int kFlagSegStart = 1 << 12; // first tile of a segment
// bits 13-15: pieces of the segment's row (0 = more than 7); bits 16-18: the
// segment's index among them (segment-start items)
constexpr int kPartsShift = 13, kPieceShift = 16;

// R = rows per TMA box: 16, or 8 for 8-token blocks (two boxes per tile).
template <int D, int HG, int NS, int R>
struct Layout {
  static constexpr int kHalves = D / 64;
  static constexpr int kRegion = R * 128;                 // one (head, half) box slice
  static constexpr int kBox = HG * kHalves * kRegion;     // one box, K or V
  static constexpr int kSide = kBox * (kTile / R);        // K (or V) of one tile
  static constexpr int kStage = 2 * kSide;
  static constexpr int off_desc = NS * kStage;
  static constexpr int off_bar = off_desc + NS * 16;  // full[NS], empty[NS], qfree[2]
  static constexpr int off_misc = off_bar + (2 * NS + 2) * 8;
  // misc: RangeInfo (64 B) + block-scan scratch (8 B per warp, <= 9 warps);
  // then the prefixes of the sequences the dynamic tail units lie in
  static constexpr int off_tail = off_misc + 160;
  static constexpr int kTailBytes = ((kDynSeqs + 1) * 8 + kDynSeqs * 4 + 15) / 16 * 16;
  // per consumer warp: [8 heads][D + 4] fp32 output staging + 8 lse values
  static constexpr int kFlushStride = D + 4;  // padding spreads the 4 column lanes over banks
  static constexpr int kFlushFloats = 8 * kFlushStride + 8;
  static constexpr int off_flush = off_tail + kTailBytes;
  // q rows of the current and next segment: [2][HG * 8 heads][D] of T
  static constexpr int kQBuf = HG * 8 * D * 2;
  static constexpr int off_q = (off_flush + HG * kFlushFloats * 4 + 127) / 128 * 128;
  static constexpr int kBytes = off_q + 2 * kQBuf;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1 KB alignment
  // byte offset of row `tok` (0..15) of (head, half) inside one side
  static __device__ __forceinline__ int row_off(int head, int half, int tok) {
    return (tok / R) * kBox + ((head * kHalves + half) * R + tok % R) * 128;
  }
};

struct TmaParams {
  int one_box;  // 1: one 4-D box per side; 0: one 3-D box per (head, half)
  int q_bulk;   // 1: the producer stages each segment's q rows in shared memory
  int stall;    // test hook: CTA (0, 0) expects bytes that never come (wait runs out)
  int rope_smem;  // 1: the segment's RoPE cos/sin rows travel behind its q rows
};

template <typename T, int D, int HG, int NS, int R>
__global__ void __launch_bounds__(32 * (HG + 1), 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv,
                      const DecodeArgs a, const TmaParams tp) {
  using L = Layout<D, HG, NS, R>;
  constexpr int NT = 32 * (HG + 1);
  constexpr int KS = D / 16;  // k-steps of QK, m-tiles of PV
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int hg = blockIdx.x, g = blockIdx.y;
  const int kv0 = hg * HG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* empty = full + NS;
  uint64_t* qfree = empty + NS;  // [2]: consumers are done reading a q buffer
  RangeInfo* ri = reinterpret_cast<RangeInfo*>(smem + L::off_misc);
  static_assert(sizeof(RangeInfo) <= 64, "RangeInfo fits its shared-memory slot");
  int64_t* sm_scan = reinterpret_cast<int64_t*>(smem + L::off_misc + 64);
  int64_t* tailp = reinterpret_cast<int64_t*>(smem + L::off_tail);
  int* tailc = reinterpret_cast<int*>(smem + L::off_tail + (kDynSeqs + 1) * 8);
  ItemDesc* desc = reinterpret_cast<ItemDesc*>(smem + L::off_desc);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], HG);
    }
    mbar_init(&qfree[0], HG);
    mbar_init(&qfree[1], HG);
    fence_mbar_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  // Launched with programmatic dependent launch: everything above overlaps
  // the previous kernel in the stream; nothing below runs before that kernel
  // has finished and its writes are visible (no input is read earlier).
  wait_prerequisites();
  find_share<NT, T>(a, g, kv0, HG, ri, sm_scan, tailp, tailc);  // includes __syncthreads
  launch_dependents();
  const int64_t start = ri->start, end = ri->end;
  const UnitPlan up = ri->plan;
  // a CTA with no static share and no units to claim only counts itself done
  const bool idle = start >= end && up.U == 0;
  uint32_t* ctr = a.zeroed ? a.ws_ctr + 2 * hg : nullptr;

  if (idle) {
    // nothing to stream
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    const bool dyn = up.U > 0;
    const int b0 = a.B > kDynSeqs ? a.B - kDynSeqs : 0;
    int64_t ustart = start, uend = end;  // the static unit first, then claimed ones
    int unit = g;
    int b = ri->b_first;
    int64_t pb = ri->p_first;
    int seg_base = 0;
    uint32_t item = 0;
    bool abort = false;
    // a claim issued ahead: lane 0 asks for the next unit two tiles before the
    // current unit's last one is issued, so the atomic's round trip overlaps
    // them instead of stalling the ring between units
    bool have_claim = false;
    int claim = 0;
    // tiles and context length of sequence lb: shared memory for the tail
    // sequences of a dynamic plan, else the context lengths in global memory
    auto seq_tiles = [&](int lb) {
      return (dyn && lb >= b0) ? static_cast<int>(tailp[lb - b0 + 1] - tailp[lb - b0])
                               : tiles_of(a, lb);
    };
    auto seq_ctx = [&](int lb) {
      return (dyn && lb >= b0) ? tailc[lb - b0] : clamp_ctx(a.context_lens[lb], a);
    };
    while (!abort) {
      if (ustart >= uend) {
        if (!dyn) break;
        int u = claim;
        if (!have_claim && lane == 0) u = static_cast<int>(atomicAdd(ctr, 1u));
        have_claim = false;
        u = __shfl_sync(kFull, u, 0);
        if (u >= up.U) break;  // every unit is taken
        unit = up.Gs + u;
        ustart = unit_start(up, unit);
        uend = unit_start(up, unit + 1);
        // the sequence holding ustart, among the last kDynSeqs sequences
        const int nt = a.B - b0;
        const bool hit = lane < nt && tailp[lane] <= ustart && ustart < tailp[lane + 1];
        const unsigned m = __ballot_sync(kFull, hit);
        if (m == 0u) {  // cannot happen with a consistent plan; never stream blind
          if (lane == 0) set_err(a.err, IR_DEVERR_CONTEXT_LEN);
          abort = true;
          break;
        }
        const int i = __ffs(m) - 1;
        b = b0 + i;
        pb = tailp[i];
      }
      int nb = seq_tiles(b);
      for (int64_t t = ustart; t < uend && !abort;) {
        const int64_t tt = t + lane;
        const bool active = tt < uend;
        int lb = b, ln = nb;
        int64_t lp = pb;
        if (active) {
          while (tt >= lp + ln) {
            lp += ln;
            ++lb;
            ln = seq_tiles(lb);
          }
        }
        const int j = static_cast<int>(tt - lp);
        const int tok0 = j * kTile;
        int packed = 0;
        int64_t row0 = 0, row1 = -1;
        bool seg_start = false;
        if (active) {
          const int ctx = seq_ctx(lb);
          const int nvalid = min(kTile, ctx - tok0);
          const int32_t* btr = a.block_tables + lb * a.bt_stride;
          bool ok;
          if (R == 8) {
            const int blk = tok0 >> 3;
            const int id0 = btr[blk];
            ok = id0 >= 0 && id0 < a.num_blocks;
            row0 = static_cast<int64_t>(id0) * 8;
            if (nvalid > 8) {
              const int id1 = btr[blk + 1];
              ok = ok && id1 >= 0 && id1 < a.num_blocks;
              row1 = static_cast<int64_t>(id1) * 8;
            }
          } else {
            const int blk = tok0 / a.bs;
            const int id0 = btr[blk];
            ok = id0 >= 0 && id0 < a.num_blocks;
            row0 = static_cast<int64_t>(id0) * a.bs + (tok0 - blk * a.bs);
          }
          if (!ok) set_err(a.err, IR_DEVERR_BLOCK_ID);
          seg_start = (tt == ustart) || (j == 0);
          const bool whole = (lp >= ustart) && (lp + ln <= uend);
          packed = nvalid | (ok ? kFlagValid : 0) | (j == ln - 1 ? kFlagSeqEnd : 0) |
                   (whole ? kFlagWhole : 0) | (seg_start ? kFlagSegStart : 0);
          if (seg_start && !whole && a.inline_merge) {
            const int u_first = unit_of(up, lp);
            const int parts = unit_of(up, lp + ln - 1) - u_first + 1;
            const int pidx = unit - u_first;
            packed |= ((parts <= 7 ? parts : 0) << kPartsShift) |
                      ((pidx < 7 ? pidx : 7) << kPieceShift);
          }
        }
        const unsigned starts = __ballot_sync(kFull, active && seg_start);
        const unsigned le_mask = (lane == 31) ? kFull : ((2u << lane) - 1u);
        const int seg = seg_base + __popc(starts & le_mask) - 1;
        const int nact = (uend - t) < 32 ? static_cast<int>(uend - t) : 32;
        const int claim_at = (dyn && t + nact >= uend) ? (nact >= 2 ? nact - 2 : 0) : -1;
        for (int k = 0; k < nact; ++k) {
          if (k == claim_at && !have_claim) {
            if (lane == 0) claim = static_cast<int>(atomicAdd(ctr, 1u));
            have_claim = true;
          }
          const uint32_t slot = item % NS;
          const uint32_t par = ((item / NS) & 1u) ^ 1u;
          int ok_wait = 1;
          if (lane == 0) ok_wait = mbar_wait_bounded(&empty[slot], par) ? 1 : 0;
          ok_wait = __shfl_sync(kFull, ok_wait, 0);
          if (!ok_wait) {
            if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
            abort = true;
            break;
          }
          const int kb = __shfl_sync(kFull, lb, k);
          const int ktok = __shfl_sync(kFull, tok0, k);
          const int kseg = __shfl_sync(kFull, seg, k);
          const int kpk = __shfl_sync(kFull, packed, k);
          const int64_t kr0 = __shfl_sync(kFull, row0, k);
          const int64_t kr1 = __shfl_sync(kFull, row1, k);
          // a segment's first tile also brings the segment's q rows (buffer
          // seg & 1), once the consumers have loaded segment seg - 2's q
          const bool with_q = tp.q_bulk && (kpk & kFlagSegStart);
          if (with_q && kseg >= 2) {
            int okq = 1;
            if (lane == 0)
              okq = mbar_wait_bounded(&qfree[kseg & 1], ((kseg >> 1) + 1) & 1) ? 1 : 0;
            if (!__shfl_sync(kFull, okq, 0)) {
              if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
              abort = true;
              break;
            }
          }
          if (lane == 0) {
            desc[slot] = ItemDesc{kb, ktok, (unit << 1) | (kseg & 1), kpk};
            uint8_t* kd = smem + slot * L::kStage;
            uint8_t* vd = kd + L::kSide;
            const uint32_t qrows = static_cast<uint32_t>(HG * a.n_rep * D * 2);
            const uint32_t qbytes = with_q ? qrows + (tp.rope_smem ? D * 8u : 0u) : 0u;
            const bool valid = (kpk & kFlagValid) != 0;
            const int nbox = (R == 8 && kr1 < 0) ? 1 : kTile / R;
            const uint32_t tbytes = valid ? static_cast<uint32_t>(nbox * 2 * L::kBox) : 0u;
            const uint32_t never = (tp.stall && item == 0 && g == 0 && hg == 0) ? 16u : 0u;
            if (valid || with_q)
              mbar_arrive_expect_tx(&full[slot], tbytes + qbytes + never);
            else
              mbar_arrive(&full[slot]);  // invalid tile: nothing to wait for
            if (with_q) {
              const T* qsrc = reinterpret_cast<const T*>(a.q) + kb * a.q_stride +
                              static_cast<int64_t>(kv0 * a.n_rep) * D;
              uint8_t* qdst = smem + L::off_q + (kseg & 1) * L::kQBuf;
              bulk_load(qdst, qsrc, qrows, &full[slot]);
              if (tp.rope_smem) {
                bulk_load(qdst + qrows, a.rope_cos + kb * a.rope_stride, D * 4, &full[slot]);
                bulk_load(qdst + qrows + D * 4, a.rope_sin + kb * a.rope_stride, D * 4,
                          &full[slot]);
              }
            }
            if (valid) {
              for (int bx = 0; bx < nbox; ++bx) {
                const int row = static_cast<int>(bx == 0 ? kr0 : kr1);
                if (tp.one_box) {
                  tma_load_4d(kd + bx * L::kBox, &tmk, &full[slot], 0, row, 0, kv0);
                  tma_load_4d(vd + bx * L::kBox, &tmv, &full[slot], 0, row, 0, kv0);
                } else {
  #pragma unroll
                  for (int h = 0; h < HG; ++h) {
  #pragma unroll
                    for (int hf = 0; hf < L::kHalves; ++hf) {
                      const int off = bx * L::kBox + (h * L::kHalves + hf) * L::kRegion;
                      tma_load_3d(kd + off, &tmk, &full[slot], 64 * hf, kv0 + h, row);
                      tma_load_3d(vd + off, &tmv, &full[slot], 64 * hf, kv0 + h, row);
                    }
                  }
                }
              }
            }
          }
          ++item;
        }
        if (abort) break;
        const int last = nact - 1;
        b = __shfl_sync(kFull, lb, last);
        pb = __shfl_sync(kFull, lp, last);
        nb = __shfl_sync(kFull, ln, last);
        seg_base += __popc(starts);
        t += nact;
      }
      ustart = uend;  // this unit is issued
    }
    if (!abort) {
      const uint32_t slot = item % NS;
      const uint32_t par = ((item / NS) & 1u) ^ 1u;
      if (lane == 0) {
        if (mbar_wait_bounded(&empty[slot], par)) {
          desc[slot] = ItemDesc{0, 0, 0, kFlagEnd};
          mbar_arrive(&full[slot]);
        } else {
          set_err(a.err, IR_DEVERR_TIMEOUT);
        }
      }
    }
  } else {
  // -------------------------------------------------------------- consumers
  const int head = warp - 1;  // 0..HG-1
  const int kvh = kv0 + head;
  const int grp = lane >> 2;      // token row / head column of fragments
  const int qd = (lane & 3) * 2;  // column pair inside fragments
  // per-lane row offsets (bytes, within one side) of the ldmatrix reads
  const int ktok = (lane & 7) + ((lane >> 3) & 1) * 8;  // K: non-transposed
  const int kcsel = lane >> 4;
  const int vtok = (lane & 7) + (lane >> 4) * 8;         // V: transposed
  const int vcsel = (lane >> 3) & 1;
  int koff[L::kHalves], voff[L::kHalves];
#pragma unroll
  for (int hf = 0; hf < L::kHalves; ++hf) {
    koff[hf] = L::row_off(head, hf, ktok);
    voff[hf] = L::row_off(head, hf, vtok);
  }

  float acc[KS][4];
  float m[2], l[2];
  uint32_t qf[KS][2];
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    qf[i][0] = qf[i][1] = 0u;
  }
  m[0] = m[1] = -INFINITY;
  l[0] = l[1] = 0.f;
  int seg_b = -1, seg_unit = 0, seg_parts = 0, seg_pidx = 0;
  bool seg_whole = false, have_seg = false;

  float* fbuf = reinterpret_cast<float*>(smem + L::off_flush) + head * L::kFlushFloats;

  // This warp has just written piece seg_pidx of the row set (kvh, seg_b),
  // which has seg_parts pieces in units seg_unit - seg_pidx, ...: count it;
  // the warp that writes the last one folds the pieces in unit order (as the
  // merge kernel does), writes the final rows and sets the counter back.
  auto merge_inline = [&]() {
    uint32_t* cnt = a.ws_seq + static_cast<int64_t>(kvh) * a.B + seg_b;
    __threadfence();  // every lane's part of this piece is visible before it is counted
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atomicAdd(cnt, 1u);
    old = __shfl_sync(kFull, old, 0);
    if (old != static_cast<uint32_t>(seg_parts - 1)) return;
    __threadfence();  // the other pieces' writes happened before their counts
    const int nr = a.n_rep;
    const int64_t base = static_cast<int64_t>(kvh) * a.ws_slots + (seg_unit - seg_pidx) + seg_b;
    const bool act = lane * 4 < D;
    for (int n = 0; n < nr; ++n) {
      float li[kInlineMax];
      float4 oi[kInlineMax];
#pragma unroll
      for (int i = 0; i < kInlineMax; ++i) {  // independent loads, one round trip
        li[i] = -INFINITY;
        oi[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < seg_parts) {
          const int64_t sl = base + i;
          li[i] = __ldcg(a.ws_lse + sl * nr + n);
          if (act) oi[i] = __ldcg(reinterpret_cast<const float4*>(a.ws_o + (sl * nr + n) * D) + lane);
        }
      }
      float M = -INFINITY, S = 0.f;
      float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < kInlineMax; ++i) {
        if (li[i] == -INFINITY) continue;
        const float Mn = fmaxf(M, li[i]);
        const float c = ex2(M - Mn), w = ex2(li[i] - Mn);
        S = S * c + w;
        r.x = r.x * c + w * oi[i].x;
        r.y = r.y * c + w * oi[i].y;
        r.z = r.z * c + w * oi[i].z;
        r.w = r.w * c + w * oi[i].w;
        M = Mn;
      }
      const bool empty_row = S == 0.f;
      const float inv = empty_row ? 0.f : 1.f / S;
      const int h = kvh * nr + n;
      if (a.lse_mode) {
        if (act)
          reinterpret_cast<float4*>(a.lse_o + (static_cast<int64_t>(seg_b) * a.H + h) * D)[lane] =
              make_float4(r.x * inv, r.y * inv, r.z * inv, r.w * inv);
        if (lane == 0)
          a.lse_out[static_cast<int64_t>(seg_b) * a.H + h] =
              empty_row ? -INFINITY : (M + log2f(S)) * kLn2;
      } else if (act) {
        T* dst = reinterpret_cast<T*>(a.out) + seg_b * a.out_stride + static_cast<int64_t>(h) * D;
        uint2 v;
        v.x = pack2<T>(r.x * inv, r.y * inv);
        v.y = pack2<T>(r.z * inv, r.w * inv);
        reinterpret_cast<uint2*>(dst)[lane] = v;
      }
    }
    __syncwarp();
    if (lane == 0) atomicExch(cnt, 0u);
  };

  // Write this warp's finished segment: the final row or a workspace piece.
  // The normalised fragments go through shared memory so that the global
  // writes are whole 16-byte pieces of contiguous head rows.
  auto flush = [&]() {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      l[j] += __shfl_xor_sync(kFull, l[j], 4);
      l[j] += __shfl_xor_sync(kFull, l[j], 8);
      l[j] += __shfl_xor_sync(kFull, l[j], 16);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const bool empty_seg = (m[j] == -INFINITY);
      const float inv = empty_seg ? 0.f : 1.f / l[j];
      float* row = fbuf + (qd + j) * L::kFlushStride;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        row[16 * i + grp] = acc[i][j] * inv;
        row[16 * i + grp + 8] = acc[i][j + 2] * inv;
      }
      if (grp == 0) fbuf[8 * L::kFlushStride + qd + j] = empty_seg ? -INFINITY : m[j] + log2f(l[j]);
    }
    __syncwarp();
    const int nr = a.n_rep;
    const float* lse2 = fbuf + 8 * L::kFlushStride;
    if (seg_whole && !a.lse_mode) {
      // final rows in T: 16-byte pieces of 8 elements
      constexpr int kPer = D / 8;
      T* dst = reinterpret_cast<T*>(a.out) + seg_b * a.out_stride +
               static_cast<int64_t>(kvh * nr) * D;
      for (int c = lane; c < nr * kPer; c += 32) {
        const int n = c / kPer, d = (c % kPer) * 8;
        const float4 x = *reinterpret_cast<const float4*>(fbuf + n * L::kFlushStride + d);
        const float4 y = *reinterpret_cast<const float4*>(fbuf + n * L::kFlushStride + d + 4);
        uint4 v;
        v.x = pack2<T>(x.x, x.y);
        v.y = pack2<T>(x.z, x.w);
        v.z = pack2<T>(y.x, y.y);
        v.w = pack2<T>(y.z, y.w);
        *reinterpret_cast<uint4*>(dst + n * D + d) = v;
      }
    } else {
      // fp32 rows: the LSE-mode output or a workspace piece
      float* dst;
      float* ldst;
      if (seg_whole) {
        dst = a.lse_o + (static_cast<int64_t>(seg_b) * a.H + kvh * nr) * D;
        ldst = a.lse_out + static_cast<int64_t>(seg_b) * a.H + kvh * nr;
      } else {
        const int64_t slot = static_cast<int64_t>(kvh) * a.ws_slots + seg_unit + seg_b;
        dst = a.ws_o + slot * nr * D;
        ldst = a.ws_lse + slot * nr;
      }
      constexpr int kPer = D / 4;
      for (int c = lane; c < nr * kPer; c += 32) {
        const int n = c / kPer, d = (c % kPer) * 4;
        *reinterpret_cast<float4*>(dst + n * D + d) =
            *reinterpret_cast<const float4*>(fbuf + n * L::kFlushStride + d);
      }
      if (lane < nr) ldst[lane] = seg_whole ? lse2[lane] * kLn2 : lse2[lane];
      if (!seg_whole && a.inline_merge && seg_parts >= 2 && seg_parts <= kInlineMax)
        merge_inline();
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < KS; ++i)
      acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
  };

  for (uint32_t item = 0;; ++item) {
    const uint32_t slot = item % NS, par = (item / NS) & 1u;
    const bool ok = mbar_wait_bounded(&full[slot], par);
    if (__any_sync(kFull, !ok)) {
      if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
      break;
    }
    const ItemDesc dsc = desc[slot];
    const int pk = dsc.packed;
    if ((pk & (kFlagSegStart | kFlagEnd)) && have_seg) flush();
    if (pk & kFlagEnd) break;
    const int b = dsc.b;
    if (pk & kFlagSegStart) {
      have_seg = true;
      seg_b = b;
      seg_unit = dsc.seg >> 1;
      seg_whole = (pk & kFlagWhole) != 0;
      seg_parts = (pk >> kPartsShift) & 7;
      seg_pidx = (pk >> kPieceShift) & 7;
      // this segment's q as B fragments: from the staged rows, else global
      const T* qrow = tp.q_bulk
          ? reinterpret_cast<const T*>(smem + L::off_q + (dsc.seg & 1) * L::kQBuf) +
                head * a.n_rep * D
          : reinterpret_cast<const T*>(a.q) + b * a.q_stride +
                static_cast<int64_t>(kvh * a.n_rep) * D;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        if (grp < a.n_rep) {
          qf[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + grp * D + 16 * ks + qd);
          qf[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + grp * D + 16 * ks + 8 + qd);
        } else {
          qf[ks][0] = qf[ks][1] = 0u;
        }
      }
      if (a.rope_cos != nullptr && grp < a.n_rep) {
        // RoPE on the q fragments: element d (column pair qd of k-step ks)
        // pairs with d + D/2, which this lane holds in k-step ks + KS/2
        const float* cs = tp.rope_smem
            ? reinterpret_cast<const float*>(
                  smem + L::off_q + (dsc.seg & 1) * L::kQBuf + HG * a.n_rep * D * 2)
            : a.rope_cos + b * a.rope_stride;
        const float* sn = tp.rope_smem ? cs + D : a.rope_sin + b * a.rope_stride;
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
#pragma unroll
          for (int w = 0; w < 2; ++w) {
            const int d = 16 * ks + 8 * w + qd;
            const float2 lo = unpack2<T>(qf[ks][w]);
            const float2 hi = unpack2<T>(qf[ks + KS / 2][w]);
            const int u = d + D / 2;
            qf[ks][w] = pack2<T>(rope_elem<T>(lo.x, hi.x, cs[d], sn[d], false),
                                 rope_elem<T>(lo.y, hi.y, cs[d + 1], sn[d + 1], false));
            qf[ks + KS / 2][w] = pack2<T>(rope_elem<T>(hi.x, lo.x, cs[u], sn[u], true),
                                          rope_elem<T>(hi.y, lo.y, cs[u + 1], sn[u + 1], true));
          }
        }
      }
      if (tp.q_bulk) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&qfree[dsc.seg & 1]);
      }
    }
    const int nvalid = (pk & kFlagValid) ? (pk & 0xff) : 0;
    uint8_t* kst = smem + slot * L::kStage;
    uint8_t* vst = kst + L::kSide;
    const uint32_t kb = smem_u32(kst);
    const uint32_t vb = kb + L::kSide;
    bool wrote = false;
    if (nvalid > 0) {
      if (nvalid < kTile) {
        // rows past the context: zero this head's V so 0 * garbage cannot make NaN
        const int per_row = L::kHalves * 8;
        for (int idx = lane; idx < (kTile - nvalid) * per_row; idx += 32) {
          const int r = nvalid + idx / per_row, rem = idx % per_row;
          *reinterpret_cast<uint4*>(vst + L::row_off(head, rem >> 3, r) + (rem & 7) * 16) =
              make_uint4(0, 0, 0, 0);
        }
        wrote = true;
      }
      if (a.k_new != nullptr && (pk & kFlagSeqEnd)) {
        // fused cache write: this tile holds position ctx-1 of sequence b
        const int r = nvalid - 1;
        const int pos = dsc.tok0 + r;
        constexpr int kChunks = D * 2 / 16;  // 16-byte chunks per row
        const int64_t slot_w = a.slot_mapping[b];
        const int32_t* btr = a.block_tables + b * a.bt_stride;
        const int64_t want = static_cast<int64_t>(btr[pos / a.bs]) * a.bs + pos % a.bs;
        if (lane == 0 && slot_w != want) set_err(a.err, IR_DEVERR_WRITE_SLOT);
        if (lane == 0 && slot_w >= a.num_slots) set_err(a.err, IR_DEVERR_SLOT);
        if (lane < 2 * kChunks) {
          const bool is_v = lane >= kChunks;
          const int c = is_v ? lane - kChunks : lane;
          const T* src = reinterpret_cast<const T*>(is_v ? a.v_new : a.k_new) +
                         b * a.kv_stride + static_cast<int64_t>(kvh) * D + c * 8;
          uint4 val = *reinterpret_cast<const uint4*>(src);
          if (!is_v && a.rope_cos != nullptr) {
            // RoPE on the new K row: chunk c pairs with chunk c ^ (kChunks / 2)
            const int pc = c ^ (kChunks / 2);
            const bool upper = c >= kChunks / 2;
            const uint4 pv = *reinterpret_cast<const uint4*>(src + (pc - c) * 8);
            const float* cs = a.rope_cos + b * a.rope_stride + c * 8;
            const float* sn = a.rope_sin + b * a.rope_stride + c * 8;
            uint32_t* xv = reinterpret_cast<uint32_t*>(&val);
            const uint32_t* yv = reinterpret_cast<const uint32_t*>(&pv);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 x = unpack2<T>(xv[e]), y = unpack2<T>(yv[e]);
              xv[e] = pack2<T>(rope_elem<T>(x.x, y.x, cs[2 * e], sn[2 * e], upper),
                               rope_elem<T>(x.y, y.y, cs[2 * e + 1], sn[2 * e + 1], upper));
            }
          }
          uint8_t* base = is_v ? vst : kst;
          *reinterpret_cast<uint4*>(base + L::row_off(head, c >> 3, r) +
                                    (((c & 7) ^ (r & 7)) << 4)) = val;
          if (slot_w >= 0 && slot_w < a.num_slots) {
            T* dst = const_cast<T*>(reinterpret_cast<const T*>(is_v ? a.v_pool : a.k_pool)) +
                     (slot_w * a.Hkv + kvh) * D + c * 8;
            *reinterpret_cast<uint4*>(dst) = val;
          }
        }
        wrote = true;
      }
      __syncwarp();

      // S^T = K . Q^T : 16 tokens x 8 head columns (two accumulators halve
      // the dependent MMA chain)
      float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const int chunk = (ks & 3) * 2 + kcsel;
        const uint32_t addr = kb + koff[ks >> 2] + ((chunk ^ (ktok & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(addr, a0, a1, a2, a3);
        if (ks & 1)
          mma_16816<T>(s2, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        else
          mma_16816<T>(s, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) s[r] += s2[r];
      // online softmax over this tile's tokens, per head column
      const bool v0 = grp < nvalid, v1 = grp + 8 < nvalid;
      float p[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float s0 = v0 ? s[j] * a.scale_log2 : -INFINITY;
        const float s1 = v1 ? s[j + 2] * a.scale_log2 : -INFINITY;
        float mx = fmaxf(s0, s1);
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, 16));
        const float mnew = fmaxf(m[j], mx);
        const float muse = (mnew == -INFINITY) ? 0.f : mnew;
        const float alpha = ex2(m[j] - muse);
        p[j] = ex2(s0 - muse);
        p[j + 2] = ex2(s1 - muse);
        l[j] = l[j] * alpha + p[j] + p[j + 2];
        m[j] = mnew;
#pragma unroll
        for (int i = 0; i < KS; ++i) {
          acc[i][j] *= alpha;
          acc[i][j + 2] *= alpha;
        }
      }
      const uint32_t pb0 = movmatrix_trans(pack2<T>(p[0], p[1]));
      const uint32_t pb1 = movmatrix_trans(pack2<T>(p[2], p[3]));
      // O^T += V^T . P^T
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        const int chunk = (i & 3) * 2 + vcsel;
        const uint32_t addr = vb + voff[i >> 2] + ((chunk ^ (vtok & 7)) << 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(addr, a0, a1, a2, a3);
        mma_16816<T>(acc[i], a0, a1, a2, a3, pb0, pb1);
      }
    }
    if (wrote) fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
  }  // consumers
  // every warp of the CTA is done (pieces written and merged): count the CTA
  // done; the last CTA of the kv-head group leaves the header counters at
  // zero for the next call (every exit path, aborted ones included, comes
  // through here)
  if (ctr != nullptr) {
    __syncthreads();
    if (warp == 0) {
      uint32_t old = 0;
      if (lane == 0) {
        __threadfence();
        old = atomicAdd(ctr + 1, 1u);
      }
      old = __shfl_sync(kFull, old, 0);
      if (old == gridDim.y - 1) {
        __threadfence();
        if (a.inline_merge)
          for (int i = lane; i < HG * a.B; i += 32) a.ws_seq[static_cast<int64_t>(kv0) * a.B + i] = 0u;
        if (lane == 0) {
          atomicExch(ctr, 0u);
          atomicExch(ctr + 1, 0u);
        }
      }
    }
  }
}

// Stage ring depth: as many tiles as fit in one CTA's shared memory next to
// the flush buffers (one CTA per SM; measured faster on B200 than two CTAs
// with half the stages each). IRB_TMA_STAGES caps it for tuning builds.
#ifndef IRB_TMA_STAGES
#define IRB_TMA_STAGES 16
#endif
template <int D, int HG, int R>
constexpr int stages_for() {
  constexpr int stage = 2 * HG * (D / 64) * kTile * 128;  // K + V of one tile
  constexpr int flush = HG * (8 * (D + 4) + 8) * 4;
  constexpr int qbuf = 2 * HG * 8 * D * 2;
  constexpr int tail = ((kDynSeqs + 1) * 8 + kDynSeqs * 4 + 15) / 16 * 16;
  constexpr int budget = 227 * 1024 - 1024 - 672 - tail - flush - qbuf;  // align slack, misc
  constexpr int fit = budget / (stage + 48);                // + desc and barriers
  constexpr int n = fit < IRB_TMA_STAGES ? fit : IRB_TMA_STAGES;
  return n < 2 ? 2 : n;
}

template <typename T, int D, int HG, int R>
int launch_t(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
             const TmaParams& tp, cudaStream_t stream) {
  constexpr int NS = stages_for<D, HG, R>();
  using L = Layout<D, HG, NS, R>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = decode_tma_kernel<T, D, HG, NS, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kAlloc);
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv / HG, a.G);
  cfg.blockDim = dim3(32 * (HG + 1));
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, tmk, tmv, a, tp));
}

template <typename T, int D, int HG, int R>
int occupancy_t() {
  constexpr int NS = stages_for<D, HG, R>();
  using L = Layout<D, HG, NS, R>;
  auto kern = decode_tma_kernel<T, D, HG, NS, R>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc) !=
      cudaSuccess)
    return 1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 32 * (HG + 1), L::kAlloc) !=
      cudaSuccess)
    return 1;
  return n > 0 ? n : 1;
}

// Dispatch over (D, HG, R) for one dtype; op 0 = launch, 1 = occupancy.
template <typename T, int D, int HG>
int by_rows(int op, int R, const CUtensorMap* tmk, const CUtensorMap* tmv,
            const DecodeArgs* a, const TmaParams* tp, cudaStream_t s) {
  if (R == 8)
    return op ? occupancy_t<T, D, HG, 8>() : launch_t<T, D, HG, 8>(*tmk, *tmv, *a, *tp, s);
  return op ? occupancy_t<T, D, HG, 16>() : launch_t<T, D, HG, 16>(*tmk, *tmv, *a, *tp, s);
}

template <typename T, int D>
int by_group(int op, int HG, int R, const CUtensorMap* tmk, const CUtensorMap* tmv,
             const DecodeArgs* a, const TmaParams* tp, cudaStream_t s) {
  switch (HG) {
    case 1: return by_rows<T, D, 1>(op, R, tmk, tmv, a, tp, s);
    case 2: return by_rows<T, D, 2>(op, R, tmk, tmv, a, tp, s);
    case 4: return by_rows<T, D, 4>(op, R, tmk, tmv, a, tp, s);
    default: return by_rows<T, D, 8>(op, R, tmk, tmv, a, tp, s);
  }
}

template <typename T>
int by_dim(int op, int D, int HG, int R, const CUtensorMap* tmk, const CUtensorMap* tmv,
           const DecodeArgs* a, const TmaParams* tp, cudaStream_t s) {
  return D == 128 ? by_group<T, 128>(op, HG, R, tmk, tmv, a, tp, s)
                  : by_group<T, 64>(op, HG, R, tmk, tmv, a, tp, s);
}

}  // namespace

int tma_head_group(int num_kv_heads) {
  for (int hg : {8, 4, 2, 1})
    if (num_kv_heads % hg == 0) return hg;
  return 1;
}

int launch_decode_tma(const CUtensorMap& tmk, const CUtensorMap& tmv, const DecodeArgs& a,
                      int dtype, int one_box, int stall, cudaStream_t stream) {
  // q rows of a head group move as one bulk copy when 16-byte aligned
  const int64_t grp_elems = static_cast<int64_t>(a.n_rep) * a.D;
  const bool q_ok = (reinterpret_cast<uintptr_t>(a.q) % 16 == 0) && (a.q_stride * 2) % 16 == 0 &&
                    (grp_elems * 2) % 16 == 0;
  const int HG = tma_head_group(a.Hkv), R = a.bs == 8 ? 8 : 16;
  // RoPE rows ride in the q buffer's unused tail ([HG][8][D] of 16-bit
  // elements, HG * n_rep rows used) when 16-byte aligned and it has room
  const bool rope_smem = q_ok && a.rope_cos != nullptr &&
                         reinterpret_cast<uintptr_t>(a.rope_cos) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(a.rope_sin) % 16 == 0 &&
                         (a.rope_stride * 4) % 16 == 0 &&
                         static_cast<int64_t>(HG) * (8 - a.n_rep) * a.D * 2 >= 8 * a.D;
  const TmaParams tp{one_box, q_ok ? 1 : 0, stall, rope_smem ? 1 : 0};
  if (dtype == IR_DTYPE_BF16)
    return by_dim<__nv_bfloat16>(0, a.D, HG, R, &tmk, &tmv, &a, &tp, stream);
  return by_dim<__half>(0, a.D, HG, R, &tmk, &tmv, &a, &tp, stream);
}

int decode_tma_occupancy(int dtype, int D, int Hkv, int bs) {
  const int HG = tma_head_group(Hkv), R = bs == 8 ? 8 : 16;
  if (dtype == IR_DTYPE_BF16)
    return by_dim<__nv_bfloat16>(1, D, HG, R, nullptr, nullptr, nullptr, nullptr, nullptr);
  return by_dim<__half>(1, D, HG, R, nullptr, nullptr, nullptr, nullptr, nullptr);
}

}  // namespace irb
