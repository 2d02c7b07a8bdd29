// Paged prefill / mixed-varlen attention on the 5th-generation tensor cores.
//
// Query rows are packed: sequence s owns rows [q_start[s], q_start[s+1]),
// which are its last q_len positions ctx - q_len .. ctx - 1; the row at
// position p attends the sequence's positions 0..p, read through its block
// table from the paged K/V pool (the causal / varlen masks of
// infrared/model/inputs.py:38-94 applied to infrared's paged read).
//
// One CTA = 128 query rows of one sequence for one query head (grid:
// q tiles x heads). Six warps:
//   warp 4      producer: TMA copies of the Q tile (once) and of each
//               128-key K tile and V tile (one 16-row box per 16-slot block
//               and 64-column half) into rings of NS stages;
//   warp 5      MMA issuer (one thread): S = Q.K^T (M=128, N=128 keys,
//               K=D) into one of two TMEM buffers, then O_tile = P.V
//               (M=128, N=D, K=128 keys) into a third, tcgen05.mma
//               kind::f16 with operands in 128-byte-swizzled shared memory;
//               tcgen05.commit releases stages and signals the softmax;
//   warps 0-3   softmax (thread r = query row r = TMEM lane r): row max of
//               the masked scores, exp2 probabilities written as 16-bit P
//               into shared memory (the A operand of the P.V MMA), running
//               sum, and the fp32 output accumulated in registers from each
//               tile's O_tile (rescaled when the row max grows).
// The QK^T MMA of tile j+1 runs while the softmax works on tile j.
// Every wait is bounded (2 s); on a timeout the CTA flags IR_DEVERR_TIMEOUT,
// lets its copies and MMAs drain (bounded), frees its tensor memory and ends.
#include "tcgen05.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kRows = 128;     // query rows per CTA (MMA M)
constexpr int kKeys = 128;     // keys per K/V tile
constexpr int kThreads = 192;  // warps 0-3 softmax, 4 producer, 5 MMA
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;  // S buffers at columns 0 and 128, O_tile at 256

template <int D>
struct PLayout {
  static constexpr int kHalves = D / 64;
  static constexpr int kHalf = kRows * 128;              // one 64-column half of a tile
  static constexpr int kQ = kHalves * kHalf;             // Q tile
  static constexpr int kSide = kHalves * kKeys * 128;    // one K or V tile
  static constexpr int NS = D == 128 ? 2 : 4;            // stages per ring
  static constexpr int off_q = 0;
  static constexpr int off_k = kQ;
  static constexpr int off_v = off_k + NS * kSide;
  static constexpr int off_p = off_v + NS * kSide;       // P: 2 halves x 128 rows x 128 B
  static constexpr int kP = 2 * kHalf;
  static constexpr int off_bar = off_p + kP;
  // q_full, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS], s_full[2], s_free[2],
  // p_full, o_full, o_free, drain
  static constexpr int kBars = 1 + 4 * NS + 8;
  static constexpr int off_misc = off_bar + kBars * 8;
  static constexpr int kBytes = off_misc + 64;
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

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap tmq,
                      const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv, const PrefillArgs a) {
  using L = PLayout<D>;
  constexpr int NS = L::NS;
  constexpr bool kBf16 = DT<T>::code == IR_DTYPE_BF16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + NS;
  uint64_t* v_full = k_empty + NS;
  uint64_t* v_empty = v_full + NS;
  uint64_t* s_full = v_empty + NS;  // [2]
  uint64_t* s_free = s_full + 2;    // [2]
  uint64_t* p_full = s_free + 2;
  uint64_t* o_full = p_full + 1;
  uint64_t* o_free = o_full + 1;
  uint64_t* drain = o_free + 1;
  int* misc = reinterpret_cast<int*>(smem + L::off_misc);  // seq, tile, tmem base
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;

  if (warp == 0) {
    int sq, tl;
    locate_tile(a, blockIdx.x, lane, &sq, &tl);
    if (lane == 0) {
      misc[0] = sq;
      misc[1] = tl;
    }
  }
  if (threadIdx.x == 32) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kRows);
    }
    mbar_init(p_full, kRows);
    mbar_init(o_full, 1);
    mbar_init(o_free, kRows);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 64) {
    prefetch_tensormap(&tmq);
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  __syncthreads();
  const int s = misc[0];
  if (s < 0) return;
  const int qt = misc[1];
  const int qs = a.q_start[s];
  const int ql = a.q_start[s + 1] - qs;
  int ctx = a.context_lens[s];
  const int maxc = a.max_blocks * a.bs;
  if (ctx < ql || ctx > maxc) {
    if (threadIdx.x == 0) set_err(a.err, IR_DEVERR_CONTEXT_LEN);
    return;
  }
  const int r0 = qs + qt * kRows;
  const int nrows = min(kRows, ql - qt * kRows);
  const int pos0 = ctx - ql + qt * kRows;  // position of row 0
  const int n_kv = (pos0 + nrows - 1) / kKeys + 1;
  const int kvh = h / a.n_rep;

  if (warp == 0) tc::alloc(reinterpret_cast<uint32_t*>(&misc[2]), kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = static_cast<uint32_t>(misc[2]);

  if (warp == 4) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, L::kQ);
#pragma unroll
      for (int hf = 0; hf < L::kHalves; ++hf)
        tma_load_3d(smem + L::off_q + hf * L::kHalf, &tmq, q_full, 64 * hf, h, r0);
      const int R = a.bs < kKeys ? a.bs : kKeys;  // rows per box
      const int nbox = kKeys / R;
      const int32_t* btr = a.block_tables + static_cast<int64_t>(s) * a.bt_stride;
      const int oob = static_cast<int>(a.num_slots);  // zero-filled by the copy
      int issued = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % NS;
        const uint32_t par = ((j / NS) & 1) ^ 1;
        // rows of the tile's blocks (out-of-range coordinates read zeros)
        auto row_of = [&](int i) {
          const int key0 = j * kKeys + i * R;
          if (key0 >= ctx) return oob;
          const int id = btr[key0 / a.bs];
          if (id < 0 || id >= a.num_blocks) {
            set_err(a.err, IR_DEVERR_BLOCK_ID);
            return oob;
          }
          return id * a.bs + key0 % a.bs;
        };
        if (!mbar_wait_bounded(&k_empty[st], par)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], L::kSide);
        uint8_t* kd = smem + L::off_k + st * L::kSide;
        for (int i = 0; i < nbox; ++i) {
          const int row = row_of(i);
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
            tma_load_3d(kd + hf * (kKeys * 128) + i * R * 128, &tmk, &k_full[st], 64 * hf, kvh,
                        row);
        }
        if (!mbar_wait_bounded(&v_empty[st], par)) {
          ok = false;
          // the K copies of this tile are in flight: count it as issued
          issued = j + 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::kSide);
        uint8_t* vd = smem + L::off_v + st * L::kSide;
        for (int i = 0; i < nbox; ++i) {
          const int row = row_of(i);
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
            tma_load_3d(vd + hf * (kKeys * 128) + i * R * 128, &tmv, &v_full[st], 64 * hf, kvh,
                        row);
        }
        issued = j + 1;
      }
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // no copy may still be writing when the CTA ends
      mbar_wait_bounded(q_full, 0);
      for (int j = issued > NS ? issued - NS : 0; j < issued; ++j) {
        mbar_wait_bounded(&k_full[j % NS], (j / NS) & 1);
        if (ok || j + 1 < issued) mbar_wait_bounded(&v_full[j % NS], (j / NS) & 1);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait_bounded(q_full, 0);
      const uint32_t qb = smem_u32(smem + L::off_q);
      const uint32_t pb = smem_u32(smem + L::off_p);
      constexpr uint32_t kIdS = tc::idesc_f16(kRows, kKeys, kBf16, false);
      constexpr uint32_t kIdO = tc::idesc_f16(kRows, D, kBf16, true);
      auto issue_qk = [&](int j) -> bool {
        const int st = j % NS, sb = j & 1;
        if (!mbar_wait_bounded(&k_full[st], (j / NS) & 1)) return false;
        if (!mbar_wait_bounded(&s_free[sb], ((j >> 1) & 1) ^ 1)) return false;
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
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j % NS;
        if (!mbar_wait_bounded(&v_full[st], (j / NS) & 1)) return false;
        if (!mbar_wait_bounded(p_full, j & 1)) return false;
        if (!mbar_wait_bounded(o_free, (j & 1) ^ 1)) return false;
        tc::fence_after_sync();
        const uint32_t vb = smem_u32(smem + L::off_v + st * L::kSide);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          const uint32_t po = (k >> 2) * L::kHalf + (k & 3) * 32;
          tc::mma_f16_ss(tmem + kColO, tc::sw128_desc(pb + po, 16, 1024),
                         tc::sw128_desc(vb + k * 2048, kKeys * 128, 1024), kIdO, k > 0);
        }
        tc::commit(o_full);
        tc::commit(&v_empty[st]);
        return true;
      };
      if (ok) ok = issue_qk(0);
      for (int j = 0; j < n_kv && ok; ++j) {
        if (j + 1 < n_kv) ok = issue_qk(j + 1);
        if (ok) ok = issue_pv(j);
      }
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // every MMA issued has completed before the tensor memory is freed
      tc::commit(drain);
      mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------------------------------------------------- softmax
    const int r = threadIdx.x;  // query row = TMEM lane
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int pos = pos0 + r;
    const int lim = min(pos, ctx - 1);  // last key this row may attend
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    uint8_t* prow = smem + L::off_p + (r >> 3) * 1024 + (r & 7) * 128;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      const int kbase = j * kKeys;
      // tcgen05.ld is warp-collective: a warp leaves the loop as a whole
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&s_full[sb], (j >> 1) & 1))) {
        ok = false;
        break;
      }
      tc::fence_after_sync();
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKeys / 32; ++c) {
        float v[32];
        tc::ld32(lane_addr + sb * kKeys + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (kbase + c * 32 + i <= lim) mx = fmaxf(mx, v[i]);
      }
      const float m_new = fmaxf(m, mx * a.scale_log2);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = ex2(m - m_use);
      if (j > 0) {
        // tile j-1's P.V: O = O * alpha_{j-1} + O_tile
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(o_full, (j - 1) & 1))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          tc::ld32(lane_addr + kColO + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha_prev, v[i]);
        }
        tc::fence_before_sync();
        mbar_arrive(o_free);
      }
      // probabilities of tile j -> P (16-bit, swizzled K-major rows)
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kKeys / 32; ++c) {
        float v[32];
        tc::ld32(lane_addr + sb * kKeys + c * 32, v);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int key = kbase + c * 32 + i;
          const float p0 = key <= lim ? ex2(fmaf(v[i], a.scale_log2, -m_use)) : 0.f;
          const float p1 = key + 1 <= lim ? ex2(fmaf(v[i + 1], a.scale_log2, -m_use)) : 0.f;
          sum += p0 + p1;
          pk[i >> 1] = pack2<T>(p0, p1);
        }
        uint8_t* hrow = prow + (c >> 1) * L::kHalf;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int ch = ((c & 1) * 4 + k) ^ (r & 7);
          *reinterpret_cast<uint4*>(hrow + ch * 16) =
              make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
        }
      }
      if (j == n_kv - 1 && kbase + r >= ctx) {
        // key row r of the last tile lies past the context: zero its V row so
        // that 0 * (stale pool bits) cannot reach the output
        if (mbar_wait_bounded(&v_full[j % NS], (j / NS) & 1)) {
          uint8_t* vrow = smem + L::off_v + (j % NS) * L::kSide + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
#pragma unroll
            for (int k = 0; k < 8; ++k)
              *reinterpret_cast<uint4*>(vrow + hf * (kKeys * 128) + k * 16) =
                  make_uint4(0, 0, 0, 0);
        } else {
          ok = false;
        }
      }
      fence_proxy_async_shared();
      tc::fence_before_sync();
      mbar_arrive(p_full);
      mbar_arrive(&s_free[sb]);
      l = fmaf(l, alpha, sum);
      m = m_new;
      alpha_prev = alpha;
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
    }
    if (ok) {
      if (__all_sync(0xffffffffu, mbar_wait_bounded(o_full, (n_kv - 1) & 1))) {
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          tc::ld32(lane_addr + kColO + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = fmaf(o[c * 32 + i], alpha_prev, v[i]);
        }
      } else {
        ok = false;
      }
    }
    if (!ok) {
      set_err(a.err, IR_DEVERR_TIMEOUT);
    } else if (r < nrows) {
      const float inv = 1.f / l;
      T* dst = reinterpret_cast<T*>(a.out) + static_cast<int64_t>(r0 + r) * a.out_stride +
               static_cast<int64_t>(h) * D;
#pragma unroll
      for (int d = 0; d < D; d += 8) {
        uint4 w;
        w.x = pack2<T>(o[d] * inv, o[d + 1] * inv);
        w.y = pack2<T>(o[d + 2] * inv, o[d + 3] * inv);
        w.z = pack2<T>(o[d + 4] * inv, o[d + 5] * inv);
        w.w = pack2<T>(o[d + 6] * inv, o[d + 7] * inv);
        *reinterpret_cast<uint4*>(dst + d) = w;
      }
    }
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
             const PrefillArgs& a, int tiles, cudaStream_t stream) {
  using L = PLayout<D>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = prefill_tc_kernel<T, D>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc);
  if (e != cudaSuccess) return static_cast<int>(e);
  kern<<<dim3(tiles, a.H), kThreads, L::kAlloc, stream>>>(tmq, tmk, tmv, a);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

int launch_prefill_tc(const CUtensorMap& tmq, const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const PrefillArgs& a, int dtype, cudaStream_t stream) {
  // an upper bound of the q tiles: every sequence adds at most one partial tile
  const int tiles = (a.total_q + kRows - 1) / kRows + a.S;
  if (tiles == 0 || a.H == 0) return 0;
  if (dtype == IR_DTYPE_BF16)
    return a.D == 128 ? launch_t<__nv_bfloat16, 128>(tmq, tmk, tmv, a, tiles, stream)
                      : launch_t<__nv_bfloat16, 64>(tmq, tmk, tmv, a, tiles, stream);
  return a.D == 128 ? launch_t<__half, 128>(tmq, tmk, tmv, a, tiles, stream)
                    : launch_t<__half, 64>(tmq, tmk, tmv, a, tiles, stream);
}

}  // namespace irb
