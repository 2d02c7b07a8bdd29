// Exchange of KV-chunk partials between the GPUs of one node over NVLink,
// with peer stores instead of a collective library call, in ONE kernel.
//
// Every rank owns one exchange buffer (cudaMalloc'd, zeroed once, mapped into
// every peer process with CUDA IPC):
//   header  epoch u32 (offset 0)   calls this rank has completed
//           done  u32 (offset 64)  exchange CTAs finished (monotonic)
//   slots   [2 parities][world sources][rows][D/2 + 1] chunks of 16 bytes
// A chunk is {x, flag, y, flag}: two fp32 values of a row (the last chunk of a
// row holds its lse) and, twice, the flag of the call that wrote it
// (call index + 1). A 16-byte store reaches the peer's memory as one unit
// (each 8-byte half at least), so a reader that sees the flag in both halves
// of a chunk also sees that call's values there: no fences and no arrival
// counters, one NVLink trip from store to use (the "LL" idea of NCCL's
// low-latency protocol, in a layout of this file's own).
//
// Call n on rank r (n = r's epoch; parity n & 1): each warp takes rows
// row = warp_id, warp_id + total_warps, ...; it first stores r's (o, lse) of
// all its rows into slot [n & 1][r] of every peer's buffer, then polls the
// chunks of the same rows from every peer in its own buffer until their flags
// read n + 1, and combines the world's partials in rank order (ir_lse_merge's
// arithmetic, so every rank writes identical rows). The last CTA to finish
// advances the epoch.
//
// Forward progress: a warp waits only for rows that the warp with the same
// index on each peer stores before it waits for anything, and the grid is at
// most one CTA per SM (a 128-thread CTA with no shared-memory demand), so
// every CTA of every rank is resident at once and no wait depends on a CTA
// that cannot be scheduled. The grid is a function of the buffer's row
// capacity and the SM count only, so it is the same on every call on a
// buffer, which the epoch counter relies on.
//
// Slot layout: rows are placed by the buffer's row capacity (from its size),
// not by the call's row count, so calls with fewer rows (a smaller batch)
// use the same slots; every rank must allocate the same size.
//
#include "common.cuh"
#include "decode_common.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kHeader = 4096;
constexpr int kEpoch = 0, kDone = 64;
constexpr int kWarps = 16;  // rows are spread over the warps of at most one CTA per SM
constexpr int kThreads = 32 * kWarps;

__device__ __forceinline__ void st_chunk(uint8_t* p, float x, float y, uint32_t flag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p),
               "r"(__float_as_uint(x)), "r"(flag), "r"(__float_as_uint(y)), "r"(flag)
               : "memory");
}

__device__ __forceinline__ uint4 ld_chunk(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint8_t* row_slot(uint8_t* buf, const PeerArgs& p, int par, int src,
                                             int row) {
  const int64_t chunks = p.D / 2 + 1;
  return buf + kHeader +
         ((static_cast<int64_t>(par) * p.world + src) * p.cap + row) * chunks * 16;
}

// CPL = chunks (value pairs) per lane: 1 for D <= 64, 2 for D <= 128.
template <int CPL>
__device__ __forceinline__ void load_row(const float* o, const PeerArgs& p, int row, int lane,
                                         float2 (&v)[CPL]) {
  const int C = p.D / 2;
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    const int c = lane + 32 * k;
    const float* src = o + static_cast<int64_t>(row) * p.D + 2 * c;
    v[k] = c < C ? *reinterpret_cast<const float2*>(src) : make_float2(0.f, 0.f);
  }
}

template <typename T, int CPL>
__global__ void __launch_bounds__(kThreads)
    exchange_kernel(T* __restrict__ out, int64_t out_stride, const float* __restrict__ o,
                    const float* __restrict__ lse, int H, const PeerArgs p) {
  __shared__ uint32_t s_n;
  uint8_t* own = p.bufs[p.rank];
  launch_dependents();   // the next kernel may run its prologue while this one waits
  wait_prerequisites();  // o / lse come from the kernel before this one
  if (threadIdx.x == 0) s_n = *reinterpret_cast<volatile uint32_t*>(own + kEpoch);
  __syncthreads();
  const uint32_t n = s_n, flag = n + 1;
  const int par = n & 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int first = blockIdx.x * kWarps + warp;
  const int step = gridDim.x * kWarps;
  const int C = p.D / 2;
  // 1. this rank's partial of every row of the warp, into every peer's buffer
  for (int row = first; row < p.rows; row += step) {
    float2 mine[CPL];
    load_row<CPL>(o, p, row, lane, mine);
    const float my_lse = lse[row];
    for (int q = 0; q < p.world; ++q) {
      if (q == p.rank) continue;
      uint8_t* dst = row_slot(p.bufs[q], p, par, p.rank, row);
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        const int c = lane + 32 * k;
        if (c < C) st_chunk(dst + c * 16, mine[k].x, mine[k].y, flag);
      }
      if (lane == 0) st_chunk(dst + C * 16, my_lse, 0.f, flag);
    }
  }
  // 2. every source's rows (this rank's from its own o / lse), merged in rank
  // order; a source whose wait ran out once is left out of the warp's later
  // rows, so a silent peer costs one wait limit per warp, not one per row
  unsigned missing = 0;
  for (int row = first; row < p.rows; row += step) {
    float l_src[8];
    float2 v_src[8][CPL];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      l_src[s] = -INFINITY;
      if (s >= p.world || ((missing >> s) & 1u)) continue;
      if (s == p.rank) {
        l_src[s] = lse[row];
        load_row<CPL>(o, p, row, lane, v_src[s]);
        continue;
      }
      const uint8_t* src = row_slot(own, p, par, s, row);
      unsigned long long t0 = 0;
      int spins = 0;
      while (true) {
        bool ok = true;
        uint4 ch[CPL];
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          const int c = lane + 32 * k;
          if (c < C) {
            ch[k] = ld_chunk(src + c * 16);
            ok = ok && ch[k].y == flag && ch[k].w == flag;
          } else {
            ch[k] = make_uint4(0u, flag, 0u, flag);
          }
        }
        const uint4 cl = ld_chunk(src + C * 16);
        ok = ok && cl.y == flag && cl.w == flag;
        if (__all_sync(0xffffffffu, ok)) {
          l_src[s] = __uint_as_float(cl.x);
#pragma unroll
          for (int k = 0; k < CPL; ++k)
            v_src[s][k] = make_float2(__uint_as_float(ch[k].x), __uint_as_float(ch[k].z));
          break;
        }
        if (++spins == 64) t0 = globaltimer_ns();
        if (spins > 64) {
          // lane 0's clock decides for the whole warp
          const bool out_of_time =
              __shfl_sync(0xffffffffu, globaltimer_ns() - t0 > kWaitLimitNs, 0);
          if (out_of_time) {
            if (lane == 0) set_err(p.err, IR_DEVERR_TIMEOUT);
            missing |= 1u << s;
            l_src[s] = -INFINITY;  // leave the missing partial out
            break;
          }
          __nanosleep(32);
        }
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < 8; ++s)
      if (s < p.world) M = fmaxf(M, l_src[s]);
    T* dst = out + static_cast<int64_t>(row / H) * out_stride + static_cast<int64_t>(row % H) * p.D;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = lane + 32 * k;
      if (c >= C) continue;
      float vx = 0.f, vy = 0.f;
      if (M != -INFINITY) {
        float lsum = 0.f, ox = 0.f, oy = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          if (s >= p.world || l_src[s] == -INFINITY) continue;
          const float w = ex2((l_src[s] - M) * kLog2e);
          lsum += w;
          ox += w * v_src[s][k].x;
          oy += w * v_src[s][k].y;
        }
        vx = ox / lsum;
        vy = oy / lsum;
      }
      dst[2 * c] = DT<T>::from_f(vx);
      dst[2 * c + 1] = DT<T>::from_f(vy);
    }
  }
  // the last CTA of this call advances the epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(reinterpret_cast<uint32_t*>(own + kDone), 1u);
    if (old == (n + 1) * gridDim.x - 1) *reinterpret_cast<volatile uint32_t*>(own + kEpoch) = n + 1;
  }
}

template <typename T>
int launch_t(void* out, int64_t out_stride, const float* o, const float* lse, int H,
             const PeerArgs& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  // the same grid on every call on a buffer: the epoch protocol counts this
  // kernel's CTAs per call
  cfg.gridDim = dim3(peer_exchange_grid(p.cap, p.sms));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  T* dst = static_cast<T*>(out);
  const cudaError_t e = p.D <= 64
                            ? cudaLaunchKernelEx(&cfg, exchange_kernel<T, 1>, dst, out_stride, o,
                                                 lse, H, p)
                            : cudaLaunchKernelEx(&cfg, exchange_kernel<T, 2>, dst, out_stride, o,
                                                 lse, H, p);
  return static_cast<int>(e);
}

}  // namespace

size_t peer_exchange_bytes(int world, int rows, int D) {
  return kHeader + static_cast<size_t>(2) * world * rows * (D / 2 + 1) * 16;
}

int64_t peer_exchange_capacity(size_t bytes, int world, int D) {
  if (bytes <= static_cast<size_t>(kHeader)) return 0;
  return static_cast<int64_t>((bytes - kHeader) /
                              (static_cast<size_t>(2) * world * (D / 2 + 1) * 16));
}

int peer_exchange_grid(int64_t cap, int sms) {
  const int64_t need = (cap + kWarps - 1) / kWarps;
  const int64_t g = need < sms ? need : sms;
  return static_cast<int>(g < 1 ? 1 : g);
}

int launch_peer_exchange(void* out, int64_t out_stride, const float* o, const float* lse, int H,
                         int dtype, const PeerArgs& p, cudaStream_t s) {
  if (p.rows == 0) return 0;
  switch (dtype) {
    case IR_DTYPE_F32: return launch_t<float>(out, out_stride, o, lse, H, p, s);
    case IR_DTYPE_BF16: return launch_t<__nv_bfloat16>(out, out_stride, o, lse, H, p, s);
    default: return launch_t<__half>(out, out_stride, o, lse, H, p, s);
  }
}

}  // namespace irb
