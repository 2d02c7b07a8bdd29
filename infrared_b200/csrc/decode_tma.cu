// Paged decode attention for 16-bit pools: TMA-fed, warp-specialised.
//
// One CTA streams one share of the 16-token tiles of one kv head (see
// decode_common.cuh). Warp 0 is the producer: its lanes resolve 32 tiles at a
// time (sequence walk + block-table lookup), then lane 0 issues, per tile,
// TMA tensor copies of the K and V rows ([16 rows x 128 B] boxes with the
// 128-byte swizzle, so the ldmatrix reads below are conflict free) into a
// ring of NS stages guarded by full/empty mbarriers. Warps 1-4 consume tiles
// round robin. Per tile a consumer warp computes, for every query head of
// the GQA group at once (padded to 8 columns):
//   S^T[16 tok x 8 heads] = K[16 x D] . Q^T[D x 8]    (D/16 mma.m16n8k16)
//   online softmax over the 16 tokens per head (exp2 on the SFU, fp32)
//   O^T[D x 8]           += V^T[D x 16] . P^T[16 x 8]  (D/16 mma.m16n8k16)
// with P^T moved into B-operand layout by two movmatrix transposes, so each
// K/V element is read from HBM once for the whole group. The tensor-core
// instructions here are the warp-level mma.sync form: the path is bound by
// HBM bandwidth, and mma.sync only removes the FMA/convert instruction issue
// that would otherwise cap a CUDA-core GEMV at ~7 FMAs per loaded element.
// At the end of each segment the four consumer warps combine their running
// (max, sum, accumulator) states through shared memory (log-sum-exp) and
// write the final row or a workspace partial.
#include "decode_common.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = 32 * (1 + kConsumerWarps);
constexpr unsigned kFull = 0xffffffffu;

struct __align__(16) ItemDesc {
  int b;
  int tok0;
  int seg;
  int packed;  // n_valid in bits 0-7, flags above
};
constexpr int kFlagValid = 1 << 8;    // copies were issued (block ids valid)
constexpr int kFlagSeqEnd = 1 << 9;   // last tile of the sequence
constexpr int kFlagWhole = 1 << 10;   // the segment is the whole sequence
constexpr int kFlagEnd = 1 << 11;     // end-of-stream marker

template <int D, int NS>
struct Layout {
  static constexpr int kHalf = kTile * 128;           // 16 rows x 128 B
  static constexpr int kHalves = D / 64;              // 64-element column halves
  static constexpr int kStage = 2 * kHalves * kHalf;  // K + V of one tile
  static constexpr int kCombStride = D * 8 + 16;      // floats per warp
  static constexpr int off_comb = NS * kStage;
  static constexpr int off_desc = off_comb + kConsumerWarps * kCombStride * 4;
  static constexpr int off_bar = off_desc + NS * 16;
  static constexpr int off_misc = off_bar + (2 * NS + 2) * 8;
  static constexpr int kBytes = off_misc + 256;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1 KB alignment
};

template <typename T, int D, int NS, bool BS8>
__global__ void __launch_bounds__(kThreads)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv,
                      const DecodeArgs a) {
  using L = Layout<D, NS>;
  constexpr int KS = D / 16;  // k-steps of QK, m-tiles of PV
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int kvh = blockIdx.x, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* empty = full + NS;
  uint64_t* flush_full = empty + NS;
  uint64_t* flush_done = flush_full + 1;
  RangeInfo* ri = reinterpret_cast<RangeInfo*>(smem + L::off_misc);
  int* seg_b = reinterpret_cast<int*>(smem + L::off_misc + 64);
  int* seg_whole = seg_b + 2;
  int64_t* sm_scan = reinterpret_cast<int64_t*>(smem + L::off_misc + 128);
  ItemDesc* desc = reinterpret_cast<ItemDesc*>(smem + L::off_desc);

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(flush_full, kConsumerWarps);
    mbar_init(flush_done, kConsumerWarps);
    fence_mbar_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  find_share<kThreads, T>(a, g, kvh, ri, sm_scan);  // includes __syncthreads
  const int64_t start = ri->start, end = ri->end;
  if (start >= end) return;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int b = ri->b_first;
    int64_t pb = ri->p_first;
    int nb = tiles_of(a, b);
    int seg_base = 0;
    uint32_t item = 0;
    bool abort = false;
    for (int64_t t = start; t < end && !abort;) {
      const int64_t tt = t + lane;
      const bool active = tt < end;
      int lb = b, ln = nb;
      int64_t lp = pb;
      if (active) {
        while (tt >= lp + ln) {
          lp += ln;
          ++lb;
          ln = tiles_of(a, lb);
        }
      }
      const int j = static_cast<int>(tt - lp);
      const int tok0 = j * kTile;
      int packed = 0;
      int64_t row0 = 0, row1 = -1;
      bool seg_start = false;
      if (active) {
        const int ctx = clamp_ctx(a.context_lens[lb], a);
        const int nvalid = min(kTile, ctx - tok0);
        const int32_t* btr = a.block_tables + lb * a.bt_stride;
        bool ok;
        if (BS8) {
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
        seg_start = (tt == start) || (j == 0);
        const bool whole = (lp >= start) && (lp + ln <= end);
        packed = nvalid | (ok ? kFlagValid : 0) |
                 (j == ln - 1 ? kFlagSeqEnd : 0) | (whole ? kFlagWhole : 0);
      }
      const unsigned starts = __ballot_sync(kFull, active && seg_start);
      const unsigned le_mask = (lane == 31) ? kFull : ((2u << lane) - 1u);
      const int seg = seg_base + __popc(starts & le_mask) - 1;
      const int nact = (end - t) < 32 ? static_cast<int>(end - t) : 32;
      for (int k = 0; k < nact; ++k) {
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
        if (lane == 0) {
          desc[slot] = ItemDesc{kb, ktok, kseg, kpk};
          uint8_t* st = smem + slot * L::kStage;
          uint8_t* kd = st;
          uint8_t* vd = st + L::kHalves * L::kHalf;
          if (kpk & kFlagValid) {
            if (BS8) {
              const uint32_t boxes = kr1 >= 0 ? 2u : 1u;
              mbar_arrive_expect_tx(&full[slot],
                                    boxes * 2u * L::kHalves * (8u * 128u));
#pragma unroll
              for (int h = 0; h < L::kHalves; ++h) {
                tma_load_3d(kd + h * L::kHalf, &tmk, &full[slot], 64 * h, kvh,
                            static_cast<int>(kr0));
                tma_load_3d(vd + h * L::kHalf, &tmv, &full[slot], 64 * h, kvh,
                            static_cast<int>(kr0));
                if (kr1 >= 0) {
                  tma_load_3d(kd + h * L::kHalf + 8 * 128, &tmk, &full[slot],
                              64 * h, kvh, static_cast<int>(kr1));
                  tma_load_3d(vd + h * L::kHalf + 8 * 128, &tmv, &full[slot],
                              64 * h, kvh, static_cast<int>(kr1));
                }
              }
            } else {
              mbar_arrive_expect_tx(&full[slot], L::kStage);
#pragma unroll
              for (int h = 0; h < L::kHalves; ++h) {
                tma_load_3d(kd + h * L::kHalf, &tmk, &full[slot], 64 * h, kvh,
                            static_cast<int>(kr0));
                tma_load_3d(vd + h * L::kHalf, &tmv, &full[slot], 64 * h, kvh,
                            static_cast<int>(kr0));
              }
            }
          } else {
            mbar_arrive(&full[slot]);
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
    if (!abort) {
      for (int k = 0; k < kConsumerWarps; ++k) {
        const uint32_t slot = item % NS;
        const uint32_t par = ((item / NS) & 1u) ^ 1u;
        int ok_wait = 1;
        if (lane == 0) ok_wait = mbar_wait_bounded(&empty[slot], par) ? 1 : 0;
        ok_wait = __shfl_sync(kFull, ok_wait, 0);
        if (!ok_wait) {
          if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
          break;
        }
        if (lane == 0) {
          desc[slot] = ItemDesc{0, 0, seg_base, kFlagEnd};
          mbar_arrive(&full[slot]);
        }
        ++item;
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int ct = cw * 32 + lane;  // 0..127
  float* comb_all = reinterpret_cast<float*>(smem + L::off_comb);
  float* comb = comb_all + cw * L::kCombStride;
  const int grp = lane >> 2;       // token row / head column of fragments
  const int qd = (lane & 3) * 2;   // column pair inside fragments

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
  int cur_seg = 0, cur_b = -1;
  uint32_t flushes = 0;
  bool abort = false;

  // Combine the four warps' states of segment cur_seg and write it out.
  auto flush = [&]() -> bool {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      l[j] += __shfl_xor_sync(kFull, l[j], 4);
      l[j] += __shfl_xor_sync(kFull, l[j], 8);
      l[j] += __shfl_xor_sync(kFull, l[j], 16);
    }
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      const int d0 = 16 * i + grp;
      *reinterpret_cast<float2*>(&comb[d0 * 8 + qd]) =
          make_float2(acc[i][0], acc[i][1]);
      *reinterpret_cast<float2*>(&comb[(d0 + 8) * 8 + qd]) =
          make_float2(acc[i][2], acc[i][3]);
    }
    if (lane < 4) {
      comb[D * 8 + qd] = m[0];
      comb[D * 8 + qd + 1] = m[1];
      comb[D * 8 + 8 + qd] = l[0];
      comb[D * 8 + 8 + qd + 1] = l[1];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(flush_full);
    bool ok = mbar_wait_bounded(flush_full, flushes & 1u);
    if (__any_sync(kFull, !ok)) {
      if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
      return false;
    }
    const int sb = seg_b[cur_seg & 1];
    const bool whole = seg_whole[cur_seg & 1] != 0;
    for (int idx = ct; idx < a.n_rep * D; idx += 32 * kConsumerWarps) {
      const int n = idx / D, d = idx - n * D;
      float mw[kConsumerWarps], M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        mw[w] = comb_all[w * L::kCombStride + D * 8 + n];
        M = fmaxf(M, mw[w]);
      }
      float val = 0.f, lse2 = -INFINITY;
      if (M != -INFINITY) {
        float lsum = 0.f, osum = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float wt = ex2(mw[w] - M);
          lsum += wt * comb_all[w * L::kCombStride + D * 8 + 8 + n];
          osum += wt * comb_all[w * L::kCombStride + d * 8 + n];
        }
        val = osum / lsum;
        lse2 = M + log2f(lsum);
      }
      write_segment_value<T>(a, kvh, g, sb, whole, n, d, val, lse2);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(flush_done);
    ok = mbar_wait_bounded(flush_done, flushes & 1u);
    if (__any_sync(kFull, !ok)) {
      if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
      return false;
    }
    ++flushes;
#pragma unroll
    for (int i = 0; i < KS; ++i)
      acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    m[0] = m[1] = -INFINITY;
    l[0] = l[1] = 0.f;
    return true;
  };

  for (uint32_t item = cw;; item += kConsumerWarps) {
    const uint32_t slot = item % NS, par = (item / NS) & 1u;
    const bool ok = mbar_wait_bounded(&full[slot], par);
    if (__any_sync(kFull, !ok)) {
      if (lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
      abort = true;
      break;
    }
    const ItemDesc dsc = desc[slot];
    const int pk = dsc.packed;
    while (cur_seg < dsc.seg && !abort) {
      abort = !flush();
      ++cur_seg;
    }
    if (abort || (pk & kFlagEnd)) break;

    const int b = dsc.b;
    if (lane == 0) {
      seg_b[cur_seg & 1] = b;
      seg_whole[cur_seg & 1] = (pk & kFlagWhole) ? 1 : 0;
    }
    if (b != cur_b) {
      cur_b = b;
      const T* qrow = reinterpret_cast<const T*>(a.q) + b * a.q_stride +
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
    }
    const int nvalid = (pk & kFlagValid) ? (pk & 0xff) : 0;
    uint8_t* st = smem + slot * L::kStage;
    uint8_t* vst = st + L::kHalves * L::kHalf;
    const uint32_t kb = smem_u32(st);
    const uint32_t vb = kb + L::kHalves * L::kHalf;
    bool wrote = false;
    if (nvalid > 0) {
      if (nvalid < kTile) {
        // rows past the context: zero V so 0 * garbage cannot make NaN
        const int per_row = L::kHalves * 8;
        for (int idx = lane; idx < (kTile - nvalid) * per_row; idx += 32) {
          const int r = nvalid + idx / per_row, rem = idx % per_row;
          *reinterpret_cast<uint4*>(vst + (rem >> 3) * L::kHalf + r * 128 +
                                    (rem & 7) * 16) = make_uint4(0, 0, 0, 0);
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
          const uint4 val = *reinterpret_cast<const uint4*>(src);
          uint8_t* base = is_v ? vst : st;
          const int cc = c & 7;
          *reinterpret_cast<uint4*>(base + (c >> 3) * L::kHalf + r * 128 +
                                    ((cc ^ (r & 7)) << 4)) = val;
          if (slot_w >= 0 && slot_w < a.num_slots) {
            T* dst = const_cast<T*>(reinterpret_cast<const T*>(is_v ? a.v_pool : a.k_pool)) +
                     (slot_w * a.Hkv + kvh) * D + c * 8;
            *reinterpret_cast<uint4*>(dst) = val;
          }
        }
        wrote = true;
      }
      __syncwarp();

      // S^T = K . Q^T : 16 tokens x 8 head columns
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int tok = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int csel = lane >> 4;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int chunk = (ks & 3) * 2 + csel;
          const uint32_t addr = kb + (ks >> 2) * L::kHalf + tok * 128 +
                                ((chunk ^ (tok & 7)) << 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(addr, a0, a1, a2, a3);
          mma_16816<T>(s, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        }
      }
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
      {
        const int mi = lane >> 3;
        const int tok = (lane & 7) + (mi >> 1) * 8;
        const int csel = mi & 1;
#pragma unroll
        for (int i = 0; i < KS; ++i) {
          const int chunk = (i & 3) * 2 + csel;
          const uint32_t addr = vb + (i >> 2) * L::kHalf + tok * 128 +
                                ((chunk ^ (tok & 7)) << 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_trans(addr, a0, a1, a2, a3);
          mma_16816<T>(acc[i], a0, a1, a2, a3, pb0, pb1);
        }
      }
    }
    if (wrote) fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
  }
}

template <typename T, int D, int NS, bool BS8>
int launch_one(const CUtensorMap& tmk, const CUtensorMap& tmv,
               const DecodeArgs& a, cudaStream_t stream) {
  using L = Layout<D, NS>;
  auto kern = decode_tma_kernel<T, D, NS, BS8>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  cudaError_t e = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return static_cast<int>(e);
  dim3 grid(a.Hkv, a.G);
  kern<<<grid, kThreads, L::kAlloc, stream>>>(tmk, tmv, a);
  return static_cast<int>(cudaGetLastError());
}

template <typename T, int D, int NS, bool BS8>
int occupancy_one() {
  using L = Layout<D, NS>;
  auto kern = decode_tma_kernel<T, D, NS, BS8>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::kAlloc) != cudaSuccess)
    return 1;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads,
                                                    L::kAlloc) != cudaSuccess)
    return 1;
  return n > 0 ? n : 1;
}

constexpr int kStages = 8;  // multiple of kConsumerWarps (slot reuse stays in one warp)
static_assert(kStages % kConsumerWarps == 0, "stage ring must align with warps");

template <typename T>
int dispatch_launch(const CUtensorMap& tmk, const CUtensorMap& tmv,
                    const DecodeArgs& a, cudaStream_t s) {
  const bool bs8 = a.bs == 8;
  if (a.D == 128)
    return bs8 ? launch_one<T, 128, kStages, true>(tmk, tmv, a, s)
               : launch_one<T, 128, kStages, false>(tmk, tmv, a, s);
  return bs8 ? launch_one<T, 64, kStages, true>(tmk, tmv, a, s)
             : launch_one<T, 64, kStages, false>(tmk, tmv, a, s);
}

template <typename T>
int dispatch_occupancy(int D, bool bs8) {
  if (D == 128)
    return bs8 ? occupancy_one<T, 128, kStages, true>()
               : occupancy_one<T, 128, kStages, false>();
  return bs8 ? occupancy_one<T, 64, kStages, true>()
             : occupancy_one<T, 64, kStages, false>();
}

}  // namespace

int launch_decode_tma(const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const DecodeArgs& a, int dtype, cudaStream_t stream) {
  if (dtype == IR_DTYPE_BF16)
    return dispatch_launch<__nv_bfloat16>(tmk, tmv, a, stream);
  return dispatch_launch<__half>(tmk, tmv, a, stream);
}

int decode_tma_occupancy(int dtype, int D, int bs) {
  if (dtype == IR_DTYPE_BF16)
    return dispatch_occupancy<__nv_bfloat16>(D, bs == 8);
  return dispatch_occupancy<__half>(D, bs == 8);
}

}  // namespace irb
