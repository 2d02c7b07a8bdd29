// K/V projection of a decode step's new tokens with the cache write in its
// epilogue, on the 5th-generation tensor cores.
//
// infrared's Attention.forward (infrared/model/layers.py:158-165) computes
//   k = x @ W_k^T + b_k,  v = x @ W_v^T + b_v      (nn.Linear, bf16 out)
//   k = k * cos + rotate_half(k) * sin             (apply_rotary_pos_emb)
// and paged_attention then scatters k and v into the pool by slot
// (infrared/cache/paged_kv_cache.py:48-57). Here one kernel does all of it
// for up to 128 tokens per tile: the projected rows never exist as tensors,
// they go from the accumulator to their pool slots.
//
// Decomposition: one cluster of kSplit CTAs per (128-token tile, output
// head), where the output heads are the Hkv heads of K followed by the Hkv
// heads of V (N = head_dim = 64 or 128 columns each). CTA r of the cluster
// takes the r-th slice of the hidden dimension (split-K), so a decode step's
// weights are streamed by kSplit x 2 Hkv CTAs at once:
//   warp 0, one lane: TMA copies of x [128 x 64] and W [N x 64] per stage
//                     (128-byte swizzle, a ring of kNS stages, whose shared
//                     memory then holds the partial sums);
//   warp 1, one lane: tcgen05.mma kind::f16, M = 128 tokens, N = head_dim,
//                     K = 16 per instruction, accumulating in TMEM;
//   warps 0-3:        each thread reads its token row of the accumulator and
//                     stores it in shared memory; after a cluster barrier,
//                     CTA r sums the kSplit partials of its 128 / kSplit rows
//                     in rank order (distributed shared memory; the same
//                     order every call), adds the bias, rounds to the model
//                     dtype as the projection's output, applies RoPE to K
//                     (rope_elem: the rounding sequence of PyTorch's
//                     elementwise ops) and stores the row into the pool at
//                     slot_mapping[token] in 16-byte pieces.
// Every mbarrier wait is bounded (2 s, IR_DEVERR_TIMEOUT); a CTA that gave up
// still writes a (zero) partial and reaches both cluster barriers, so no CTA
// of the cluster waits for it forever; copies in flight are drained
// (bounded) before tensor memory is freed.
#include "tcgen05.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kM = 128;        // token rows per tile (MMA M)
constexpr int kKc = 64;        // hidden elements per stage (one 128-byte row)
constexpr int kSplit = 8;      // CTAs per cluster (portable cluster size)
constexpr int kNS = 6;         // ring stages (a 3584-wide hidden is 7 chunks per CTA)
constexpr int kThreads = 128;  // 4 warps
constexpr int kRowsPer = kM / kSplit;  // rows each CTA reduces and writes

template <int D>
struct KvLayout {
  static constexpr int kStageA = kM * 128;                 // x: 128 rows x 128 B
  static constexpr int kStageB = D * 128;                  // W: D rows x 128 B
  static constexpr int kPartStride = D + 4;                // fp32 row of the partial
  static constexpr int off_a = 0;
  static constexpr int off_b = kNS * kStageA;
  // the partial sums reuse the ring once every MMA (the ring's last reader)
  // has completed
  static constexpr int off_part = 0;
  static_assert(kM * kPartStride * 4 <= kNS * (kStageA + kStageB), "partial fits the ring");
  static constexpr int off_bar = off_b + kNS * kStageB;  // full, empty, acc
  static constexpr int off_slot = off_bar + (2 * kNS + 1) * 8;
  static constexpr int kBytes = off_slot + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1 KB alignment
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 16 bytes of CTA `rank`'s shared memory at the address `local` has in this CTA.
__device__ __forceinline__ float4 ld_dsmem4(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)),
               "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    kv_proj_kernel(const __grid_constant__ CUtensorMap tmx,
                   const __grid_constant__ CUtensorMap tmwk,
                   const __grid_constant__ CUtensorMap tmwv, const KvProjArgs a) {
  using L = KvLayout<D>;
  constexpr bool kBf16 = DT<T>::code == IR_DTYPE_BF16;
  constexpr int kHalfD = D / 2;
  constexpr int kSegCols = D / 16;  // columns of each half a reducing thread owns
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* empty = full + kNS;
  uint64_t* acc = empty + kNS;  // every MMA of this CTA has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_slot);
  float* part = reinterpret_cast<float*>(smem + L::off_part);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int oh = blockIdx.y;  // output head: the K heads, then the V heads
  const bool is_k = oh < a.Hkv;
  const int kvh = is_k ? oh : oh - a.Hkv;
  const int m0 = blockIdx.z * kM;
  const CUtensorMap* tmw = is_k ? &tmwk : &tmwv;
  const int chunks = a.K / kKc;
  const int c_lo = static_cast<int>((rank * chunks) / kSplit);
  const int nck = static_cast<int>(((rank + 1) * chunks) / kSplit) - c_lo;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc, 1);
    fence_mbar_init();
  }
  if (threadIdx.x == 32) {
    prefetch_tensormap(&tmx);
    prefetch_tensormap(tmw);
  }
  if (warp == 0) tc::alloc(tmem_slot, D);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int i = 0;
    for (; i < nck; ++i) {
      const int st = i % kNS;
      if (!mbar_wait_bounded(&empty[st], ((i / kNS) & 1) ^ 1)) {
        set_err(a.err, IR_DEVERR_TIMEOUT);
        break;
      }
      mbar_arrive_expect_tx(&full[st], L::kStageA + L::kStageB);
      const int k0 = (c_lo + i) * kKc;
      tma_load_2d(smem + L::off_a + st * L::kStageA, &tmx, &full[st], k0, m0);
      tma_load_2d(smem + L::off_b + st * L::kStageB, tmw, &full[st], k0, kvh * D);
    }
    // no copy may still be writing when the CTA ends
    for (int j = i > kNS ? i - kNS : 0; j < i; ++j)
      mbar_wait_bounded(&full[j % kNS], (j / kNS) & 1);
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t kId = tc::idesc_f16(kM, D, kBf16, false);
    for (int i = 0; i < nck; ++i) {
      const int st = i % kNS;
      if (!mbar_wait_bounded(&full[st], (i / kNS) & 1)) {
        set_err(a.err, IR_DEVERR_TIMEOUT);
        break;
      }
      tc::fence_after_sync();
      const uint32_t ab = smem_u32(smem + L::off_a + st * L::kStageA);
      const uint32_t bb = smem_u32(smem + L::off_b + st * L::kStageB);
#pragma unroll
      for (int k = 0; k < kKc / 16; ++k)
        tc::mma_f16_ss(tmem, tc::sw128_desc(ab + k * 32, 16, 1024),
                       tc::sw128_desc(bb + k * 32, 16, 1024), kId, i > 0 || k > 0);
      tc::commit(&empty[st]);
    }
    tc::commit(acc);  // arrives once the MMAs above complete (at once if none ran)
  }
  __syncwarp();

  // this thread's rows and columns of the reduction, and the epilogue inputs
  // for them, loaded while the MMAs finish
  const int rl = threadIdx.x / 8, seg = threadIdx.x % 8;
  const int r = static_cast<int>(rank) * kRowsPer + rl;  // row of the tile
  const int m = m0 + r;                                  // token
  const int c0 = seg * kSegCols;
  float blo[kSegCols], bhi[kSegCols], clo[kSegCols], chi[kSegCols], slo[kSegCols],
      shi[kSegCols];
  const bool rope = is_k && a.cos != nullptr;
  int64_t slot = -1;
  if (m < a.M) {
    const T* bias = reinterpret_cast<const T*>(is_k ? a.bias_k : a.bias_v);
    const float* cs = rope ? a.cos + static_cast<int64_t>(m) * a.rope_stride : nullptr;
    const float* sn = rope ? a.sin + static_cast<int64_t>(m) * a.rope_stride : nullptr;
#pragma unroll
    for (int j = 0; j < kSegCols; ++j) {
      blo[j] = bias ? DT<T>::to_f(bias[kvh * D + c0 + j]) : 0.f;
      bhi[j] = bias ? DT<T>::to_f(bias[kvh * D + kHalfD + c0 + j]) : 0.f;
      clo[j] = rope ? cs[c0 + j] : 0.f;
      chi[j] = rope ? cs[kHalfD + c0 + j] : 0.f;
      slo[j] = rope ? sn[c0 + j] : 0.f;
      shi[j] = rope ? sn[kHalfD + c0 + j] : 0.f;
    }
    slot = a.slots[m];
  }

  // ------------------------------------------- partial rows -> shared memory
  // one decision per warp: tcgen05.ld is executed by all lanes or none
  const bool done = __all_sync(0xffffffffu, mbar_wait_bounded(acc, 0));
  if (!done && lane == 0) set_err(a.err, IR_DEVERR_TIMEOUT);
  const bool have = done && nck > 0;
  tc::fence_after_sync();
  {
    const int row = warp * 32 + lane;  // = TMEM lane
    float* prow = part + row * L::kPartStride;
#pragma unroll
    for (int c = 0; c < D; c += 32) {
      float v[32];
      if (have) {
        tc::ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c, v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(prow + c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    }
  }
  cluster_sync();

  // ------------------- sum the kSplit partials of this CTA's rows, write them
  {
    float lo[kSegCols], hi[kSegCols];
#pragma unroll
    for (int j = 0; j < kSegCols; ++j) lo[j] = hi[j] = 0.f;
    const float* src = part + r * L::kPartStride;
    // all kSplit loads in flight at once; the sums still run in rank order
#pragma unroll
    for (uint32_t cta = 0; cta < static_cast<uint32_t>(kSplit); ++cta) {
#pragma unroll
      for (int q = 0; q < kSegCols; q += 4) {
        const float4 x = ld_dsmem4(src + c0 + q, cta);
        const float4 y = ld_dsmem4(src + kHalfD + c0 + q, cta);
        lo[q] += x.x; lo[q + 1] += x.y; lo[q + 2] += x.z; lo[q + 3] += x.w;
        hi[q] += y.x; hi[q + 1] += y.y; hi[q + 2] += y.z; hi[q + 3] += y.w;
      }
    }
    if (m < a.M) {
      float ylo[kSegCols], yhi[kSegCols];
#pragma unroll
      for (int j = 0; j < kSegCols; ++j) {
        // the projection's output: accumulator + bias, rounded once
        ylo[j] = DT<T>::to_f(DT<T>::from_f(lo[j] + blo[j]));
        yhi[j] = DT<T>::to_f(DT<T>::from_f(hi[j] + bhi[j]));
      }
      if (rope) {
#pragma unroll
        for (int j = 0; j < kSegCols; ++j) {
          const float xl = ylo[j], xh = yhi[j];
          ylo[j] = rope_elem<T>(xl, xh, clo[j], slo[j], false);
          yhi[j] = rope_elem<T>(xh, xl, chi[j], shi[j], true);
        }
      }
      if (slot < 0 || slot >= a.num_slots) {
        set_err(a.err, IR_DEVERR_SLOT);
      } else {
        T* dst = reinterpret_cast<T*>(is_k ? a.k_pool : a.v_pool) +
                 (slot * a.Hkv + kvh) * D;
        uint32_t wl[kSegCols / 2], wh[kSegCols / 2];
#pragma unroll
        for (int j = 0; j < kSegCols / 2; ++j) {
          wl[j] = pack2<T>(ylo[2 * j], ylo[2 * j + 1]);
          wh[j] = pack2<T>(yhi[2 * j], yhi[2 * j + 1]);
        }
        if constexpr (kSegCols == 8) {
          *reinterpret_cast<uint4*>(dst + c0) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
          *reinterpret_cast<uint4*>(dst + kHalfD + c0) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
        } else {
          *reinterpret_cast<uint2*>(dst + c0) = make_uint2(wl[0], wl[1]);
          *reinterpret_cast<uint2*>(dst + kHalfD + c0) = make_uint2(wh[0], wh[1]);
        }
      }
    }
  }
  cluster_sync();  // no CTA leaves while another still reads its partial
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::dealloc(tmem, D);
}

template <typename T, int D>
int launch_t(const CUtensorMap& tmx, const CUtensorMap& tmwk, const CUtensorMap& tmwv,
             const KvProjArgs& a, cudaStream_t s) {
  using L = KvLayout<D>;
  static_assert(L::kAlloc <= 227 * 1024, "shared memory budget");
  auto kern = kv_proj_kernel<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       L::kAlloc);
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kSplit, 2 * a.Hkv, (a.M + kM - 1) / kM);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kAlloc;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, tmx, tmwk, tmwv, a));
}

}  // namespace

int launch_kv_proj(const CUtensorMap& tmx, const CUtensorMap& tmwk, const CUtensorMap& tmwv,
                   const KvProjArgs& a, int dtype, cudaStream_t s) {
  if (a.M == 0) return 0;
  if (dtype == IR_DTYPE_BF16)
    return a.D == 128 ? launch_t<__nv_bfloat16, 128>(tmx, tmwk, tmwv, a, s)
                      : launch_t<__nv_bfloat16, 64>(tmx, tmwk, tmwv, a, s);
  return a.D == 128 ? launch_t<__half, 128>(tmx, tmwk, tmwv, a, s)
                    : launch_t<__half, 64>(tmx, tmwk, tmwv, a, s);
}

}  // namespace irb
