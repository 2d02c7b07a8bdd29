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
  // q_full, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS], s_full[2], s_free[2],
  // p_full[2], p_done[2], drain
  static constexpr int kBars = 1 + 4 * NS + 9;
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
  uint64_t* s_full = v_empty + NS;  // [2] S buffer b holds tile j (j % 2 == b)
  uint64_t* s_free = s_full + 2;    // [2] the softmax has read S buffer b
  uint64_t* p_full = s_free + 2;    // [2] P buffer b written (and O rescaled)
  uint64_t* p_done = p_full + 2;    // [2] the P.V MMA reading P buffer b completed
  uint64_t* drain = p_done + 2;
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
      mbar_init(&s_free[i], kSoftmax);
      mbar_init(&p_full[i], kSoftmax);
      mbar_init(&p_done[i], 1);
    }
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

  if (warp == 8 || warp == 9) {
    // ---------------------------------------------------------- producers
    // Warp 8 fills the K ring (and loads Q), warp 9 the V ring, so K tiles
    // run ahead of the V waits. Lane i < nbox resolves box i of a tile
    // (block-table lookup) one tile ahead, so the lookups of tile j + 1
    // overlap the waits of tile j, and issues that box's copies itself.
    const bool is_k = warp == 8;
    uint64_t* full = is_k ? k_full : v_full;
    uint64_t* empty = is_k ? k_empty : v_empty;
    const CUtensorMap* tm = is_k ? &tmk : &tmv;
    uint8_t* ring = smem + (is_k ? L::off_k : L::off_v);
    bool ok = true;
    if (is_k && lane == 0) {
      mbar_arrive_expect_tx(q_full, L::kQ);
#pragma unroll
      for (int hf = 0; hf < L::kHalves; ++hf)
        tma_load_3d(smem + L::off_q + hf * L::kHalf, &tmq, q_full, 64 * hf, h, r0);
    }
    const int R = a.bs < kKeys ? a.bs : kKeys;  // rows per box
    const int nbox = kKeys / R;                 // <= 16
    const int32_t* btr = a.block_tables + static_cast<int64_t>(s) * a.bt_stride;
    const int oob = static_cast<int>(a.num_slots);  // read as zeros by the copy
    auto row_of = [&](int j) {
      if (lane >= nbox || j >= n_kv) return oob;
      const int key0 = j * kKeys + lane * R;
      if (key0 >= ctx) return oob;
      const int id = btr[key0 / a.bs];
      if (id < 0 || id >= a.num_blocks) {
        set_err(a.err, IR_DEVERR_BLOCK_ID);
        return oob;
      }
      return id * a.bs + key0 % a.bs;
    };
    int row_cur = row_of(0);
    int issued = 0;
    for (int j = 0; j < n_kv; ++j) {
      const int row_next = row_of(j + 1);
      const int st = j % NS;
      int w = 1;
      if (lane == 0) w = mbar_wait_bounded(&empty[st], ((j / NS) & 1) ^ 1) ? 1 : 0;
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
          tma_load_3d(dst + hf * (kKeys * 128), tm, &full[st], 64 * hf, kvh, row_cur);
      }
      issued = j + 1;
      row_cur = row_next;
    }
    if (lane == 0) {
      if (!ok) set_err(a.err, IR_DEVERR_TIMEOUT);
      // no copy may still be writing when the CTA ends
      if (is_k) mbar_wait_bounded(q_full, 0);
      for (int j = issued > NS ? issued - NS : 0; j < issued; ++j)
        mbar_wait_bounded(&full[j % NS], (j / NS) & 1);
    }
  } else if (warp == 10) {
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
        const int st = j % NS, b = j & 1;
        if (!mbar_wait_bounded(&v_full[st], (j / NS) & 1)) return false;
        if (!mbar_wait_bounded(&p_full[b], (j >> 1) & 1)) return false;
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
    const int r = threadIdx.x & (kRows - 1);  // query row = TMEM lane
    const int kh = threadIdx.x >> 7;          // which 64 keys of each tile
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int pos = pos0 + r;
    const int lim = min(pos, ctx - 1);  // last key this row may attend
    float* red = reinterpret_cast<float*>(smem + L::off_red);  // [2][128]
    // The two warps of a row group meet at named barrier 1 + warp % 4 (64
    // threads). They leave the tile loop together, right after such a
    // meeting whose AND of "all waits succeeded" is false, so neither can
    // wait at a barrier the other will not reach.
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
    float m_ref = -INFINITY;    // reference max of the P values (log2 units)
    float l = 0.f;              // this half's share of the row sum
    bool ok = true;
    // tcgen05.ld / st are warp-collective: every wait result is made warp-uniform
    auto wait_all = [&](uint64_t* bar, uint32_t par) {
      return __all_sync(0xffffffffu, mbar_wait_bounded(bar, par));
    };
    for (int j = 0; j < n_kv; ++j) {
      const int b = j & 1;
      const int kbase = j * kKeys + kh * 64;
      float v[64];
      if (wait_all(&s_full[b], (j >> 1) & 1)) {
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
        float t4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
        for (int i = 4; i < 64; i += 8) {
#pragma unroll
          for (int k = 0; k < 4; ++k) t4[k] = max3(t4[k], v[i + 2 * k], v[i + 2 * k + 1]);
        }
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
      // P buffer b is free once the P.V MMA of tile j - 2 has completed
      if (j >= 2 && !wait_all(&p_done[b], ((j - 2) >> 1) & 1)) ok = false;
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
          const float2 x = f2unpack(fma2(f2pack(v[c * 8 + i], v[c * 8 + i + 1]), sc2, nm2));
          const float p0 = ex2(x.x);
          const float p1 = ex2(x.y);
          s2[i >> 1] = add2(s2[i >> 1], f2pack(p0, p1));
          pk[i >> 1] = pack2<T>(p0, p1);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) * 16)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      // rows whose reference moved: O *= factor (after the P.V of tile j - 1);
      // this thread rescales its half of the columns
      bool rescale = j > 0 && __any_sync(0xffffffffu, move);
      if (rescale && !wait_all(&p_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
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
      if (j == n_kv - 1 && j * kKeys + r >= ctx && kh < L::kHalves) {
        // key row r of the last tile lies past the context: zero its V row
        // (this thread: 64-column half kh) so that 0 * (stale pool bits)
        // cannot reach the output
        if (mbar_wait_bounded(&v_full[j % NS], (j / NS) & 1)) {
          uint8_t* vrow = smem + L::off_v + (j % NS) * L::kSide + kh * (kKeys * 128) +
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
      const float sum = (u0.x + u0.y) + (u1.x + u1.y);
      l = fmaf(l, factor, sum);
      m_ref = m_new;
      // a failed wait in this tile is acted on at the next tile's meeting
    }
    // the row sum over both halves (all pairs still in step: the loop count
    // and the break points are the same for both warps of a row group)
    red[kh * kRows + r] = l;
    pair_sync();
    const float l_row = l + red[(kh ^ 1) * kRows + r];
    if (ok) {
      const int jl = n_kv - 1;
      if (wait_all(&p_done[jl & 1], (jl >> 1) & 1)) {
        tc::fence_after_sync();
        const float inv = 1.f / l_row;
        T* dst = reinterpret_cast<T*>(a.out) + static_cast<int64_t>(r0 + r) * a.out_stride +
                 static_cast<int64_t>(h) * D + kh * kDh;
#pragma unroll
        for (int c = 0; c < kDh / 32; ++c) {
          float o[32];
          tc::ld32(lane_addr + kColO + kh * kDh + c * 32, o);  // whole warp (collective)
          if (r < nrows) {
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
      } else {
        ok = false;
      }
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
