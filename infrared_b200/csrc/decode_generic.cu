// Paged decode attention on CUDA cores for every dtype/shape the TMA kernel
// does not take (fp32 pools, GQA groups of 9-16, block sizes other than 8 or a
// multiple of 16), plus the log-sum-exp merge of partials from several GPUs.
//
// The generic kernel uses the same balanced tile shares and segment outputs
// as the TMA kernel (decode_common.cuh), so one split merge serves both. A CTA
// of 128 threads walks its tiles in order: it stages the 16 K and V rows of a
// tile in shared memory (16-byte chunks gathered through the block table, the
// next tile's chunks loaded into registers while the current one computes),
// computes the 16 x group scores with fp32 dot products, updates the
// per-head online softmax (exp2 with the scale folded into log2 units) and
// accumulates P.V with each thread owning one head-dim column.
#include "decode_common.cuh"
#include "kernels.h"

namespace irb {

namespace {

constexpr int kGenThreads = 128;
constexpr int kMaxGroup = 16;

template <typename T, int D>
__global__ void __launch_bounds__(kGenThreads)
    decode_generic_kernel(const DecodeArgs a) {
  constexpr int HPT = kGenThreads / D;            // head groups per column
  constexpr int NH = (kMaxGroup + HPT - 1) / HPT;  // heads per thread
  // rows of K padded to D + 4 floats: 16-byte aligned for the vector reads
  // of the score loop, and the 8 rows one 8-lane phase reads hit distinct
  // banks
  __shared__ __align__(16) float q_s[kMaxGroup][D];
  __shared__ __align__(16) float k_s[kTile][D + 4];
  __shared__ float v_s[kTile][D];
  __shared__ float p_s[kMaxGroup][kTile];
  __shared__ float m_s[kMaxGroup], l_s[kMaxGroup], alpha_s[kMaxGroup];
  __shared__ RangeInfo ri;
  __shared__ int64_t sm_scan[kGenThreads / 32];

  const int kvh = blockIdx.x, g = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  find_share<kGenThreads, T>(a, g, kvh, 1, &ri, sm_scan);
  launch_dependents();
  const int64_t start = ri.start, end = ri.end;
  if (start >= end) return;

  const int d = tid % D, hg = tid / D;
  const T* kpool = reinterpret_cast<const T*>(a.k_pool);
  const T* vpool = reinterpret_cast<const T*>(a.v_pool);
  // K and V rows move in 16-byte chunks: thread tid owns chunks tid,
  // tid + 128, ... of each tile side, and the next tile's chunks are loaded
  // into registers before the current tile is computed, so that the loads
  // overlap the math. Pools that are not 16-byte aligned (the host sends
  // those here too) are read element by element into the same chunks.
  constexpr int EPC = 16 / static_cast<int>(sizeof(T));  // elements per chunk
  constexpr int CPR = D / EPC;                            // chunks per row
  constexpr int NCH = kTile * CPR;                        // chunks per tile side
  constexpr int CPT = (NCH + kGenThreads - 1) / kGenThreads;
  const bool vec = ((reinterpret_cast<uintptr_t>(kpool) |
                     reinterpret_cast<uintptr_t>(vpool)) & 15) == 0;
  uint4 kr[CPT], vr[CPT];
  // the sequence (tile prefix pb, nb tiles) holding a tile
  struct Cursor {
    int b;
    int64_t pb;
    int nb;
  };
  auto advance = [&](Cursor& c, int64_t t) {
    while (t >= c.pb + c.nb) {
      c.pb += c.nb;
      ++c.b;
      c.nb = tiles_of(a, c.b);
    }
  };
  // the raw chunks of tile t: zero past the context, and for the new token of
  // a fused cache write (filled in when the tile is stored)
  auto load_tile = [&](const Cursor& c, int64_t t) {
    const int tok0 = static_cast<int>(t - c.pb) * kTile;
    const int ctx = clamp_ctx(a.context_lens[c.b], a);
    const int32_t* btr = a.block_tables + c.b * a.bt_stride;
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      kr[k] = make_uint4(0, 0, 0, 0);
      vr[k] = make_uint4(0, 0, 0, 0);
      const int i = tid + k * kGenThreads;
      if (i >= NCH) continue;
      const int r = i / CPR, cc = i % CPR;
      const int pos = tok0 + r;
      if (pos >= ctx || (a.k_new != nullptr && pos == ctx - 1)) continue;
      const int id = btr[pos / a.bs];
      if (id >= 0 && id < a.num_blocks) {
        const int64_t row = static_cast<int64_t>(id) * a.bs + pos % a.bs;
        const int64_t off = (row * a.Hkv + kvh) * D + cc * EPC;
        if (vec) {
          kr[k] = *reinterpret_cast<const uint4*>(kpool + off);
          vr[k] = *reinterpret_cast<const uint4*>(vpool + off);
        } else {
          T* kt = reinterpret_cast<T*>(&kr[k]);
          T* vt = reinterpret_cast<T*>(&vr[k]);
#pragma unroll
          for (int e = 0; e < EPC; ++e) {
            kt[e] = kpool[off + e];
            vt[e] = vpool[off + e];
          }
        }
      } else if (cc == 0) {
        set_err(a.err, IR_DEVERR_BLOCK_ID);
      }
    }
  };
  // the chunks into shared memory as fp32; the new token of a fused cache
  // write comes from the inputs (RoPE applied to K when given) and is stored
  // into the pools here, by the thread that owns its chunk
  auto store_tile = [&](const Cursor& c, int64_t t) {
    const int tok0 = static_cast<int>(t - c.pb) * kTile;
    const int ctx = clamp_ctx(a.context_lens[c.b], a);
#pragma unroll
    for (int k = 0; k < CPT; ++k) {
      const int i = tid + k * kGenThreads;
      if (i >= NCH) continue;
      const int r = i / CPR, cc = i % CPR;
      T* kt = reinterpret_cast<T*>(&kr[k]);
      T* vt = reinterpret_cast<T*>(&vr[k]);
      const int pos = tok0 + r;
      if (a.k_new != nullptr && pos < ctx && pos == ctx - 1) {
        const T* kn = reinterpret_cast<const T*>(a.k_new);
        const T* vn = reinterpret_cast<const T*>(a.v_new);
        const int64_t src = c.b * a.kv_stride + static_cast<int64_t>(kvh) * D;
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
          const int col = cc * EPC + e;
          T x = kn[src + col];
          if (a.rope_cos != nullptr) {
            const int64_t rr = c.b * a.rope_stride + col;
            x = DT<T>::from_f(rope_elem<T>(DT<T>::to_f(x), DT<T>::to_f(kn[src + (col + D / 2) % D]),
                                           a.rope_cos[rr], a.rope_sin[rr], col >= D / 2));
          }
          kt[e] = x;
          vt[e] = vn[src + col];
        }
        const int id = a.block_tables[c.b * a.bt_stride + pos / a.bs];
        const int64_t sw = a.slot_mapping[c.b];
        const int64_t want = static_cast<int64_t>(id) * a.bs + pos % a.bs;
        if (cc == 0 && sw != want) set_err(a.err, IR_DEVERR_WRITE_SLOT);
        if (sw >= 0 && sw < a.num_slots) {
          const int64_t dst = (sw * a.Hkv + kvh) * D + cc * EPC;
#pragma unroll
          for (int e = 0; e < EPC; ++e) {
            const_cast<T*>(kpool)[dst + e] = kt[e];
            const_cast<T*>(vpool)[dst + e] = vt[e];
          }
        } else if (cc == 0 && sw >= a.num_slots) {
          set_err(a.err, IR_DEVERR_SLOT);
        }
      }
#pragma unroll
      for (int e = 0; e < EPC; ++e) {
        k_s[r][cc * EPC + e] = DT<T>::to_f(kt[e]);
        v_s[r][cc * EPC + e] = DT<T>::to_f(vt[e]);
      }
    }
  };
  float acc[NH];
  Cursor cur{ri.b_first, ri.p_first, tiles_of(a, ri.b_first)};
  Cursor nxt = cur;
  int cur_b = -1;
  load_tile(cur, start);
  for (int64_t t = start; t < end; ++t) {
    advance(cur, t);
    const int b = cur.b;
    const int64_t pb = cur.pb;
    const int nb = cur.nb;
    const int j = static_cast<int>(t - pb);
    const int tok0 = j * kTile;
    const int ctx = clamp_ctx(a.context_lens[b], a);
    const int nvalid = min(kTile, ctx - tok0);
    if (t == start || j == 0) {  // segment start
      if (b != cur_b) {
        cur_b = b;
        const T* qrow = reinterpret_cast<const T*>(a.q) + b * a.q_stride +
                        static_cast<int64_t>(kvh * a.n_rep) * D;
        for (int i = tid; i < a.n_rep * D; i += kGenThreads) {
          float x = DT<T>::to_f(qrow[i]);
          if (a.rope_cos != nullptr) {
            const int c = i % D, pc = (c + D / 2) % D;
            const int64_t r = b * a.rope_stride + c;
            x = rope_elem<T>(x, DT<T>::to_f(qrow[i - c + pc]), a.rope_cos[r], a.rope_sin[r],
                             c >= D / 2);
          }
          q_s[i / D][i % D] = x;
        }
      }
      if (tid < kMaxGroup) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
      }
#pragma unroll
      for (int k = 0; k < NH; ++k) acc[k] = 0.f;
    }
    // stage tile t (its chunks are in registers), then start loading t + 1
    store_tile(cur, t);
    if (t + 1 < end) {
      advance(nxt, t + 1);
      load_tile(nxt, t + 1);
    }
    __syncthreads();
    for (int i = tid; i < kTile * a.n_rep; i += kGenThreads) {
      const int r = i % kTile, n = i / kTile;
      float s = 0.f;
#pragma unroll 4
      for (int c = 0; c < D; c += 4) {
        // the same products in the same order as one element at a time
        const float4 qv = *reinterpret_cast<const float4*>(&q_s[n][c]);
        const float4 kv = *reinterpret_cast<const float4*>(&k_s[r][c]);
        s = fmaf(qv.x, kv.x, s);
        s = fmaf(qv.y, kv.y, s);
        s = fmaf(qv.z, kv.z, s);
        s = fmaf(qv.w, kv.w, s);
      }
      p_s[n][r] = r < nvalid ? s * a.scale_log2 : -INFINITY;
    }
    __syncthreads();
    for (int n = warp; n < a.n_rep; n += kGenThreads / 32) {
      const float s = lane < kTile ? p_s[n][lane] : -INFINITY;
      float mx = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = m_s[n];
      const float mnew = fmaxf(mold, mx);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      const float p = ex2(s - muse);
      float sum = p;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      const float alpha = ex2(mold - muse);
      __syncwarp();
      if (lane < kTile) p_s[n][lane] = p;
      if (lane == 0) {
        l_s[n] = l_s[n] * alpha + sum;
        m_s[n] = mnew;
        alpha_s[n] = alpha;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < NH; ++k) {
      const int n = hg + k * HPT;
      if (n < a.n_rep) {
        float x = acc[k] * alpha_s[n];
#pragma unroll
        for (int r = 0; r < kTile; ++r) x = fmaf(p_s[n][r], v_s[r][d], x);
        acc[k] = x;
      }
    }
    if (t == end - 1 || j == nb - 1) {  // segment end
      const bool whole = (pb >= start) && (pb + nb <= end);
#pragma unroll
      for (int k = 0; k < NH; ++k) {
        const int n = hg + k * HPT;
        if (n < a.n_rep) {
          const float M = m_s[n], Lsum = l_s[n];
          const bool empty = (M == -INFINITY);
          const float val = empty ? 0.f : acc[k] / Lsum;
          const float lse2 = empty ? -INFINITY : M + log2f(Lsum);
          write_segment_value<T>(a, kvh, g, b, whole, n, d, val, lse2);
        }
      }
    }
    __syncthreads();
  }
}

// Combine the pieces of the split sequences: CTA (kv head x query head in
// group, sequence) of W warps; warp w folds pieces w, w+W, ... with an online
// log-sum-exp, each lane owning 4 consecutive head-dim columns (16-byte
// loads), then the W warp states are combined through shared memory. The
// pieces' loads are independent, so a merge costs a few L2 round trips even
// when a sequence spans dozens of CTAs (W = 8 or 16 there; 4 for 4-7 pieces;
// one warp below that, so that every merge CTA of a large grid fits beside
// the decode CTAs and starts its row as soon as the decode grid ends).
template <typename T, int W>
__global__ void __launch_bounds__(32 * W) split_merge_kernel(const DecodeArgs a) {
  launch_dependents();   // the next kernel may start its own prologue now
  __shared__ float4 s_acc[W][32];
  __shared__ float s_m[W], s_s[W];
  __shared__ long long s_sum[W][3];
  const int kvh = blockIdx.x / a.n_rep, n = blockIdx.x % a.n_rep, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b0 = a.B > kDynSeqs ? a.B - kDynSeqs : 0;
  // The tile prefix this row's pieces follow from (the decode kernel's
  // ws_prefix) depends on the context lengths alone: inputs complete before
  // the decode grid let this grid start, so for batches of up to 256
  // sequences it is summed here while the decode still runs, taking a round
  // trip off the wait below (larger batches read the decode kernel's prefix
  // after the wait: most of their rows are not split, and their CTAs would
  // sum the whole batch for nothing). Every CTA waits before it returns, so
  // this grid never completes before the decode grid.
  const bool early = a.B <= 256;  // the same in every CTA of the grid
  int64_t total = 0, pb = 0, p0 = 0, nb = 0;
  // the decode kernel's units holding this row (static shares, then
  // dynamic units if any)
  int glo = 0, parts = 0;
  auto find_units = [&]() {
    if (nb <= 0) return;
    const UnitPlan up = unit_plan(total, a.G, a.dyn, a.dyn ? p0 : 0);
    glo = unit_of(up, pb);
    parts = unit_of(up, pb + nb - 1) - glo + 1;
  };
  if (early) {
    long long below = 0, below0 = 0, all = 0;
    for (int i = threadIdx.x; i < a.B; i += 32 * W) {
      const long long t = tiles_of(a, i);
      all += t;
      if (i < b) below += t;
      if (i < b0) below0 += t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      all += __shfl_xor_sync(0xffffffffu, all, o);
      below += __shfl_xor_sync(0xffffffffu, below, o);
      below0 += __shfl_xor_sync(0xffffffffu, below0, o);
    }
    if (lane == 0) {
      s_sum[warp][0] = all;
      s_sum[warp][1] = below;
      s_sum[warp][2] = below0;
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < W; ++w) {
      total += s_sum[w][0];
      pb += s_sum[w][1];
      p0 += s_sum[w][2];
    }
    nb = tiles_of(a, b);
    find_units();
  }
  wait_prerequisites();  // the decode grid's pieces and prefix are complete
  if (!early) {
    pb = a.ws_prefix[b];
    nb = a.ws_prefix[b + 1] - pb;
    total = a.ws_prefix[a.B];
    p0 = a.ws_prefix[b0];
    find_units();
  }
  if (nb <= 0) return;  // empty context: written by the decode kernel
  if (parts == 1) return;  // written whole by one unit
  if (a.inline_merge && parts <= kInlineMax) return;  // merged in the decode kernel
  const int64_t base = static_cast<int64_t>(kvh) * a.ws_slots + glo + b;
  const float* lse = a.ws_lse + base * a.n_rep + n;       // stride n_rep per piece
  const float* o = a.ws_o + (base * a.n_rep + n) * a.D;   // stride n_rep * D per piece
  const int64_t ostride = static_cast<int64_t>(a.n_rep) * a.D;
  const bool active = lane * 4 < a.D;
  float M = -INFINITY, S = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int i = warp; i < parts; i += W) {
    const float li = lse[i * a.n_rep];
    const float4 oi = active ? *reinterpret_cast<const float4*>(o + i * ostride + lane * 4)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    if (li == -INFINITY) continue;
    const float Mn = fmaxf(M, li);
    const float c = ex2(M - Mn), w = ex2(li - Mn);  // ex2(-inf) = 0 on the first piece
    S = S * c + w;
    acc.x = acc.x * c + w * oi.x;
    acc.y = acc.y * c + w * oi.y;
    acc.z = acc.z * c + w * oi.z;
    acc.w = acc.w * c + w * oi.w;
    M = Mn;
  }
  s_acc[warp][lane] = acc;
  if (lane == 0) {
    s_m[warp] = M;
    s_s[warp] = S;
  }
  __syncthreads();
  if (warp != 0) return;
  float Mt = s_m[0];
#pragma unroll
  for (int w = 1; w < W; ++w) Mt = fmaxf(Mt, s_m[w]);
  float St = 0.f;
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < W; ++w) {
    if (s_s[w] == 0.f) continue;
    const float c = ex2(s_m[w] - Mt);
    const float4 x = s_acc[w][lane];
    St += c * s_s[w];
    r.x += c * x.x;
    r.y += c * x.y;
    r.z += c * x.z;
    r.w += c * x.w;
  }
  if (!active) return;
  const bool empty = St == 0.f;
  const float inv = empty ? 0.f : 1.f / St;
  const float lse2 = empty ? -INFINITY : Mt + log2f(St);
  const float v[4] = {r.x * inv, r.y * inv, r.z * inv, r.w * inv};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    write_segment_value<T>(a, kvh, 0, b, true, n, lane * 4 + k, v[k], lse2);
}

template <typename T>
__global__ void lse_merge_kernel(T* out, int64_t out_stride, const float* o_parts,
                                 int64_t o_part_stride, const float* lse_parts,
                                 int64_t lse_part_stride, int P, int B, int H, int D) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int64_t row = static_cast<int64_t>(b) * H + h;
  float M = -INFINITY;
  for (int p = 0; p < P; ++p) M = fmaxf(M, lse_parts[p * lse_part_stride + row]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float val = 0.f;
    if (M != -INFINITY) {
      float lsum = 0.f, osum = 0.f;
      for (int p = 0; p < P; ++p) {
        const float lp = lse_parts[p * lse_part_stride + row];
        if (lp == -INFINITY) continue;
        const float w = ex2((lp - M) * kLog2e);
        lsum += w;
        osum += w * o_parts[p * o_part_stride + row * D + d];
      }
      val = osum / lsum;
    }
    out[b * out_stride + static_cast<int64_t>(h) * D + d] = DT<T>::from_f(val);
  }
}

template <typename T>
int launch_generic_t(const DecodeArgs& a, cudaStream_t s) {
  dim3 grid(a.Hkv, a.G);
  if (a.D == 128)
    decode_generic_kernel<T, 128><<<grid, kGenThreads, 0, s>>>(a);
  else
    decode_generic_kernel<T, 64><<<grid, kGenThreads, 0, s>>>(a);
  return static_cast<int>(cudaGetLastError());
}

template <typename T>
int occupancy_generic_t(int D) {
  int n = 0;
  cudaError_t e = D == 128 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                                 &n, decode_generic_kernel<T, 128>, kGenThreads, 0)
                           : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                                 &n, decode_generic_kernel<T, 64>, kGenThreads, 0);
  return (e == cudaSuccess && n > 0) ? n : 1;
}

}  // namespace

int launch_decode_generic(const DecodeArgs& a, int dtype, cudaStream_t s) {
  switch (dtype) {
    case IR_DTYPE_F32: return launch_generic_t<float>(a, s);
    case IR_DTYPE_BF16: return launch_generic_t<__nv_bfloat16>(a, s);
    default: return launch_generic_t<__half>(a, s);
  }
}

int decode_generic_occupancy(int dtype, int D) {
  switch (dtype) {
    case IR_DTYPE_F32: return occupancy_generic_t<float>(D);
    case IR_DTYPE_BF16: return occupancy_generic_t<__nv_bfloat16>(D);
    default: return occupancy_generic_t<__half>(D);
  }
}

template <typename T, int W>
int launch_merge_t(const DecodeArgs& a, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.Hkv * a.n_rep, a.B);
  cfg.blockDim = dim3(32 * W);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, split_merge_kernel<T, W>, a));
}

template <typename T>
int launch_merge_w(const DecodeArgs& a, cudaStream_t s) {
  // a sequence of average length spans about G / B shares, and the rows of
  // the last kDynSeqs sequences also hold the dynamic units: with 8 or 16 or
  // more pieces per row, 8 or 16 warps fold them in fewer rounds; with fewer
  // than 4, one warp per row (measured: C2 +1.6 %, C3 +2.3 % against 4)
  const int b = a.B > 0 ? a.B : 1;
  const int tail = b < kDynSeqs ? b : kDynSeqs;
  const int pieces = a.G / b + (a.dyn ? kDynUnitsPerCta * a.G / tail : 0);
  if (pieces >= 16) return launch_merge_t<T, 16>(a, s);
  if (pieces >= 8) return launch_merge_t<T, 8>(a, s);
  return pieces >= 4 ? launch_merge_t<T, 4>(a, s) : launch_merge_t<T, 1>(a, s);
}

int launch_split_merge(const DecodeArgs& a, int dtype, cudaStream_t s) {
  switch (dtype) {
    case IR_DTYPE_F32: return launch_merge_w<float>(a, s);
    case IR_DTYPE_BF16: return launch_merge_w<__nv_bfloat16>(a, s);
    default: return launch_merge_w<__half>(a, s);
  }
}

int launch_lse_merge(void* out, int64_t out_stride, const float* o_parts,
                     int64_t o_part_stride, const float* lse_parts,
                     int64_t lse_part_stride, int P, int B, int H, int D,
                     int dtype, cudaStream_t s) {
  dim3 grid(B, H);
  const int threads = D >= 128 ? 128 : 64;
  switch (dtype) {
    case IR_DTYPE_F32:
      lse_merge_kernel<float><<<grid, threads, 0, s>>>(
          static_cast<float*>(out), out_stride, o_parts, o_part_stride, lse_parts,
          lse_part_stride, P, B, H, D);
      break;
    case IR_DTYPE_BF16:
      lse_merge_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>(
          static_cast<__nv_bfloat16*>(out), out_stride, o_parts, o_part_stride, lse_parts,
          lse_part_stride, P, B, H, D);
      break;
    default:
      lse_merge_kernel<__half><<<grid, threads, 0, s>>>(
          static_cast<__half*>(out), out_stride, o_parts, o_part_stride, lse_parts,
          lse_part_stride, P, B, H, D);
      break;
  }
  return static_cast<int>(cudaGetLastError());
}

}  // namespace irb
