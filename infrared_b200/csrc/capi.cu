// C ABI of infrared_b200 (declared in include/infrared_b200.h).
//
// Argument validation, device-property caching, TMA descriptor encoding,
// workspace layout and kernel dispatch. Nothing here allocates or
// synchronises; every launch goes to the caller's stream.
#include <cudaTypedefs.h>

#include <map>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>

#include "decode_common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_status(int e, const char* what) {
  if (e == 0) return IR_OK;
  return fail(IR_ERR_CUDA, std::string(what) + ": " +
                               cudaGetErrorString(static_cast<cudaError_t>(e)));
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case IR_DTYPE_F32: return 4;
    case IR_DTYPE_BF16:
    case IR_DTYPE_F16: return 2;
    default: return 0;
  }
}

bool aligned(const void* p, size_t n) {
  return (reinterpret_cast<uintptr_t>(p) % n) == 0;
}

// ------------------------------------------------------------ device cache

std::mutex g_mu;
std::map<std::pair<int, int>, int> g_cache;  // (device, key) -> value
int g_forced_path = 0;
int g_one_box = 1;
int g_stall_next = 0;  // test hook: the next TMA decode launch times out on purpose

int cached(int key, int (*compute)(int), int arg, int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_cache.find({dev, key});
  if (it != g_cache.end()) {
    *out = it->second;
    return 0;
  }
  const int v = compute(arg);
  g_cache[{dev, key}] = v;
  *out = v;
  return 0;
}

int sm_count_now(int) {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 1;
}

// key encoding for the occupancy cache:
// path(2 bits) dtype(2) D==128(1) bs8(1) log2(head group)(2)
int occ_key(int path, const ir_decode_shape* s) {
  const int hg = path == 2 ? irb::tma_head_group(s->num_kv_heads) : 1;
  const int lg = hg == 8 ? 3 : hg == 4 ? 2 : hg == 2 ? 1 : 0;
  return path | (s->dtype << 2) | ((s->head_dim == 128) << 4) |
         ((s->block_size == 8) << 5) | (lg << 6);
}

int occ_compute(int key) {
  const int path = key & 3, dtype = (key >> 2) & 3, d128 = (key >> 4) & 1,
            bs8 = (key >> 5) & 1, hg = 1 << ((key >> 6) & 3);
  const int D = d128 ? 128 : 64;
  if (path == 2) return irb::decode_tma_occupancy(dtype, D, hg, bs8 ? 8 : 16);
  return irb::decode_generic_occupancy(dtype, D);
}

// CTAs per kv head (generic) or per head group (TMA) for this path.
int ctas_per_group(int path, const ir_decode_shape* s, int* out) {
  int sms = 1, occ = 1;
  int e = cached(-1, sm_count_now, 0, &sms);
  if (e) return e;
  const int key = occ_key(path, s);
  e = cached(key, occ_compute, key, &occ);
  if (e) return e;
  const int groups = path == 2 ? s->num_kv_heads / irb::tma_head_group(s->num_kv_heads)
                               : s->num_kv_heads;
  int G = (sms * occ) / groups;
  *out = G < 1 ? 1 : (G > 65535 ? 65535 : G);
  return 0;
}

// ------------------------------------------------------------ TMA encode

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// [num_slots, Hkv, D] pool viewed as (element, slot, 64-column half, head)
// — dimensions ordered so that a box of (64, rows, D/64, head_group) lands
// in shared memory as one [rows x 128 B] region per (head, half) — with the
// 128-byte swizzle. One copy moves a tile's rows for a whole head group.
bool make_pool_map4d(CUtensorMap* map, const void* pool, int64_t num_slots,
                     int hkv, int d, int dtype, int box_rows, int head_group) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(num_slots),
                              static_cast<cuuint64_t>(d / 64),
                              static_cast<cuuint64_t>(hkv)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(hkv) * d * 2, 128,
                                 static_cast<cuuint64_t>(d) * 2};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows),
                             static_cast<cuuint32_t>(d / 64),
                             static_cast<cuuint32_t>(head_group)};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == IR_DTYPE_BF16
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 4, const_cast<void*>(pool), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The same pool as a 3-D (D, Hkv, slots) map with [rows x 1 x 64] boxes:
// one copy per (head, half) of a tile.
bool make_pool_map(CUtensorMap* map, const void* pool, int64_t num_slots,
                   int hkv, int d, int dtype, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d),
                              static_cast<cuuint64_t>(hkv),
                              static_cast<cuuint64_t>(num_slots)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2,
                                 static_cast<cuuint64_t>(hkv) * d * 2};
  const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == IR_DTYPE_BF16
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 3, const_cast<void*>(pool), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A row-major [rows, cols] 16-bit matrix as a 2-D (cols, rows) map with
// {64, box_rows} boxes and the 128-byte swizzle (the K-major operand tiles of
// the tensor-core kernels).
bool make_rows_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                   int64_t row_stride, int dtype, int box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == IR_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ------------------------------------------------------------ planning

struct Plan {
  int path;     // 1 generic, 2 tma
  int G;        // CTAs per kv head
  int dyn;      // dynamic tail units (TMA path, flag set)
  int inl;      // short rows merged in the decode kernel (TMA path, flag set)
  int64_t slots;  // partial slots per kv head
  size_t ctr_off, seq_off, prefix_off, lse_off, o_off, bytes;
};

// Workspace header, at the same place in every layout (with or without the
// flags, whatever the shape) so that no call ever writes anything else there
// and the counters stay zero between calls: the counter pair {claims, CTAs
// done} of each kv-head group, then one piece counter per (kv head,
// sequence), for at most kMaxSeqCounters rows.
constexpr size_t kCtrBytes = 256;
constexpr int64_t kMaxSeqCounters = 16384;
constexpr size_t kHeaderBytes = kCtrBytes + kMaxSeqCounters * 4;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

int check_shape(const ir_decode_shape* s) {
  if (!s) return fail(IR_ERR_INVALID_ARG, "shape is null");
  if (s->batch < 0) return fail(IR_ERR_INVALID_ARG, "batch < 0");
  if (s->num_heads <= 0 || s->num_kv_heads <= 0 ||
      s->num_heads % s->num_kv_heads != 0)
    return fail(IR_ERR_INVALID_ARG,
                "num_heads must be a positive multiple of num_kv_heads");
  if (s->num_heads / s->num_kv_heads > 16)
    return fail(IR_ERR_UNSUPPORTED, "GQA group larger than 16");
  if (s->head_dim != 64 && s->head_dim != 128)
    return fail(IR_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (s->block_size <= 0) return fail(IR_ERR_INVALID_ARG, "block_size <= 0");
  if (s->max_blocks < 0) return fail(IR_ERR_INVALID_ARG, "max_blocks < 0");
  if (s->bt_stride < s->max_blocks)
    return fail(IR_ERR_INVALID_ARG, "bt_stride < max_blocks");
  const int64_t row = static_cast<int64_t>(s->num_heads) * s->head_dim;
  if (s->q_stride < row) return fail(IR_ERR_INVALID_ARG, "q_stride < H*D");
  if (s->out_stride < row) return fail(IR_ERR_INVALID_ARG, "out_stride < H*D");
  if (s->num_slots < s->block_size || s->num_slots % s->block_size != 0)
    return fail(IR_ERR_INVALID_ARG,
                "num_slots must be a positive multiple of block_size");
  if (elem_bytes(s->dtype) == 0) return fail(IR_ERR_INVALID_ARG, "bad dtype");
  if (static_cast<int64_t>(s->max_blocks) * s->block_size > INT32_MAX)
    return fail(IR_ERR_UNSUPPORTED, "max_blocks * block_size overflows int32");
  if (s->flags & ~(IR_DECODE_DYNAMIC_TAIL | IR_DECODE_INLINE_MERGE))
    return fail(IR_ERR_INVALID_ARG, "unknown bits in flags (set it to 0 or a combination "
                                    "of IR_DECODE_DYNAMIC_TAIL and IR_DECODE_INLINE_MERGE)");
  return IR_OK;
}

bool tma_eligible(const ir_decode_shape* s) {
  const int n_rep = s->num_heads / s->num_kv_heads;
  return (s->dtype == IR_DTYPE_BF16 || s->dtype == IR_DTYPE_F16) &&
         n_rep <= 8 && (s->block_size == 8 || s->block_size % 16 == 0) &&
         s->num_slots <= INT32_MAX && (s->q_stride % 2) == 0;
}

int make_plan(const ir_decode_shape* s, Plan* p) {
  int rc = check_shape(s);
  if (rc) return rc;
  int path = tma_eligible(s) ? 2 : 1;
  if (g_forced_path == 1) path = 1;
  if (g_forced_path == 2) {
    if (path != 2)
      return fail(IR_ERR_UNSUPPORTED, "TMA path forced but shape not eligible");
  }
  int G = 1;
  int e = ctas_per_group(path, s, &G);
  if (e) return cuda_status(e, "cudaGetDevice");
  p->path = path;
  p->G = G;
  const int64_t B = s->batch, H = s->num_heads, D = s->head_dim;
  const int groups = path == 2 ? s->num_kv_heads / irb::tma_head_group(s->num_kv_heads) : 0;
  const bool hdr = path == 2 && static_cast<size_t>(groups) * 8 <= kCtrBytes;
  p->dyn = (s->flags & IR_DECODE_DYNAMIC_TAIL) && hdr;
  p->inl = (s->flags & IR_DECODE_INLINE_MERGE) && hdr &&
           static_cast<int64_t>(s->num_kv_heads) * B <= kMaxSeqCounters;
  p->slots = G + (p->dyn ? static_cast<int64_t>(irb::kDynUnitsPerCta) * G : 0) + B;
  const int64_t slots = static_cast<int64_t>(s->num_kv_heads) * p->slots *
                        (H / s->num_kv_heads);
  p->ctr_off = 0;
  p->seq_off = kCtrBytes;
  p->prefix_off = kHeaderBytes;
  p->lse_off = p->prefix_off + align256(static_cast<size_t>(B + 1) * 8);
  p->o_off = p->lse_off + align256(static_cast<size_t>(slots) * 4);
  p->bytes = p->o_off + align256(static_cast<size_t>(slots * D) * 4);
  return IR_OK;
}

enum class Mode { kFinal, kLse, kWrite };

int decode_impl(Mode mode, void* out, float* lse_o, float* lse_out,
                const void* q, const void* k_pool, const void* v_pool,
                const void* k_new, const void* v_new, int64_t kv_stride,
                const int64_t* slot_mapping, const int32_t* block_tables,
                const int32_t* context_lens, const ir_decode_shape* s,
                void* workspace, size_t workspace_bytes, int32_t* err,
                cudaStream_t stream, const float* rope_cos = nullptr,
                const float* rope_sin = nullptr, int64_t rope_stride = 0) {
  Plan plan;
  int rc = make_plan(s, &plan);
  if (rc) return rc;
  if (s->batch == 0) return IR_OK;
  if (!q || !k_pool || !v_pool || !context_lens ||
      (s->max_blocks > 0 && !block_tables))
    return fail(IR_ERR_INVALID_ARG, "null input pointer");
  if (mode == Mode::kLse ? (!lse_o || !lse_out) : !out)
    return fail(IR_ERR_INVALID_ARG, "null output pointer");
  if (mode == Mode::kWrite && (!k_new || !v_new || !slot_mapping))
    return fail(IR_ERR_INVALID_ARG, "null k_new / v_new / slot_mapping");
  if (mode == Mode::kWrite && kv_stride < static_cast<int64_t>(s->num_kv_heads) * s->head_dim)
    return fail(IR_ERR_INVALID_ARG, "kv_stride < Hkv*D");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return fail(IR_ERR_INVALID_ARG, "rope_cos and rope_sin must both be given");
  if (rope_cos && (rope_stride < s->head_dim || !aligned(rope_cos, 4) || !aligned(rope_sin, 4)))
    return fail(IR_ERR_INVALID_ARG, "rope tables: stride < head_dim or not 4-byte aligned");
  if (!workspace || workspace_bytes < plan.bytes)
    return fail(IR_ERR_WORKSPACE, "workspace smaller than ir_paged_decode_workspace_size");
  if (!aligned(workspace, 256))
    return fail(IR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  const int eb = elem_bytes(s->dtype);
  if (plan.path == 2) {
    // TMA descriptors need 16-byte aligned pools; q fragments are read as
    // 32-bit words; the fused write moves 16-byte vectors.
    bool ok = aligned(k_pool, 16) && aligned(v_pool, 16) && aligned(q, 4);
    // finished rows leave in 16-byte stores (fp32 rows in LSE mode)
    if (mode == Mode::kLse)
      ok = ok && aligned(lse_o, 16);
    else
      ok = ok && aligned(out, 16) && (s->out_stride * eb) % 16 == 0;
    if (mode == Mode::kWrite)
      ok = ok && aligned(k_new, 16) && aligned(v_new, 16) &&
           (kv_stride * eb) % 16 == 0;
    if (!ok) {
      if (g_forced_path == 2)
        return fail(IR_ERR_UNSUPPORTED, "TMA path forced but pointers misaligned");
      plan.path = 1;
      // the generic path may want a different CTA count; never exceed the
      // count the workspace was sized for
      int G = 1;
      ctas_per_group(1, s, &G);
      plan.G = G > plan.G ? plan.G : G;
    }
  }
  irb::DecodeArgs a{};
  a.q = q;
  a.q_stride = s->q_stride;
  a.out = out;
  a.out_stride = s->out_stride;
  a.lse_o = lse_o;
  a.lse_out = lse_out;
  a.lse_mode = mode == Mode::kLse ? 1 : 0;
  a.block_tables = block_tables;
  a.bt_stride = s->bt_stride;
  a.context_lens = context_lens;
  a.B = s->batch;
  a.H = s->num_heads;
  a.Hkv = s->num_kv_heads;
  a.n_rep = s->num_heads / s->num_kv_heads;
  a.D = s->head_dim;
  a.bs = s->block_size;
  a.max_blocks = s->max_blocks;
  a.num_slots = s->num_slots;
  a.num_blocks = s->num_slots / s->block_size;
  a.scale_log2 = s->scale * irb::kLog2e;
  a.G = plan.G;
  a.dyn = plan.dyn && plan.path == 2 ? 1 : 0;
  a.inline_merge = plan.inl && plan.path == 2 ? 1 : 0;
  a.zeroed = a.dyn || a.inline_merge;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.ws_ctr = reinterpret_cast<uint32_t*>(ws + plan.ctr_off);
  a.ws_seq = reinterpret_cast<uint32_t*>(ws + plan.seq_off);
  a.ws_prefix = reinterpret_cast<int64_t*>(ws + plan.prefix_off);
  a.ws_slots = plan.slots;
  a.ws_lse = reinterpret_cast<float*>(ws + plan.lse_off);
  a.ws_o = reinterpret_cast<float*>(ws + plan.o_off);
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.k_new = mode == Mode::kWrite ? k_new : nullptr;
  a.v_new = mode == Mode::kWrite ? v_new : nullptr;
  a.kv_stride = kv_stride;
  a.slot_mapping = slot_mapping;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.rope_stride = rope_stride;
  a.err = err;

  int e;
  if (plan.path == 2) {
    CUtensorMap tmk, tmv;
    const int rows = s->block_size == 8 ? 8 : 16;
    const int hg = irb::tma_head_group(s->num_kv_heads);
    int one_box = g_one_box;
    if (one_box &&
        !(make_pool_map4d(&tmk, k_pool, s->num_slots, s->num_kv_heads, s->head_dim,
                          s->dtype, rows, hg) &&
          make_pool_map4d(&tmv, v_pool, s->num_slots, s->num_kv_heads, s->head_dim,
                          s->dtype, rows, hg)))
      one_box = 0;  // the driver refused the permuted view: one copy per (head, half)
    if (!one_box &&
        !(make_pool_map(&tmk, k_pool, s->num_slots, s->num_kv_heads, s->head_dim,
                        s->dtype, rows) &&
          make_pool_map(&tmv, v_pool, s->num_slots, s->num_kv_heads, s->head_dim,
                        s->dtype, rows)))
      return fail(IR_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    int stall = 0;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      stall = g_stall_next;
      g_stall_next = 0;
    }
    e = irb::launch_decode_tma(tmk, tmv, a, s->dtype, one_box, stall, stream);
  } else {
    e = irb::launch_decode_generic(a, s->dtype, stream);
  }
  if (e) return cuda_status(e, "decode kernel launch");
  e = irb::launch_split_merge(a, s->dtype, stream);
  return cuda_status(e, "merge kernel launch");
}

// ------------------------------------------------------------ prefill

int g_prefill_path = 0;  // 0 auto, 1 rows as decode rows, 2 tensor cores, 3 CTA pairs

bool make_q_map(CUtensorMap* map, const void* q, int total_q, int h, int d, int64_t q_stride,
                int dtype) {
  auto enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(h),
                              static_cast<cuuint64_t>(total_q)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(d) * 2,
                                 static_cast<cuuint64_t>(q_stride) * 2};
  const cuuint32_t box[3] = {64, 1, 128};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == IR_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 3, const_cast<void*>(q), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int check_prefill_shape(const ir_prefill_shape* s) {
  if (!s) return fail(IR_ERR_INVALID_ARG, "shape is null");
  if (s->num_seqs < 0 || s->total_q < 0) return fail(IR_ERR_INVALID_ARG, "negative size");
  if (s->num_heads <= 0 || s->num_kv_heads <= 0 || s->num_heads % s->num_kv_heads != 0)
    return fail(IR_ERR_INVALID_ARG, "num_heads must be a positive multiple of num_kv_heads");
  if (s->head_dim != 64 && s->head_dim != 128)
    return fail(IR_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (s->block_size <= 0 || s->max_blocks < 0 || s->num_slots < 0)
    return fail(IR_ERR_INVALID_ARG, "bad block_size / max_blocks / num_slots");
  if (s->bt_stride < s->max_blocks) return fail(IR_ERR_INVALID_ARG, "bt_stride < max_blocks");
  const int64_t row = static_cast<int64_t>(s->num_heads) * s->head_dim;
  if (s->q_stride < row || s->out_stride < row)
    return fail(IR_ERR_INVALID_ARG, "q_stride / out_stride < num_heads * head_dim");
  if (elem_bytes(s->dtype) == 0) return fail(IR_ERR_INVALID_ARG, "unknown dtype");
  if (static_cast<int64_t>(s->max_blocks) * s->block_size > INT32_MAX)
    return fail(IR_ERR_INVALID_ARG, "max_blocks * block_size exceeds int32");
  return IR_OK;
}

// The tensor-core kernel takes 16-bit dtypes, head_dim 64/128, power-of-two
// block sizes >= 8 and slot counts addressable by int32 copy coordinates.
bool prefill_tc_eligible(const ir_prefill_shape* s) {
  const int bs = s->block_size;
  return (s->dtype == IR_DTYPE_BF16 || s->dtype == IR_DTYPE_F16) && bs >= 8 &&
         (bs & (bs - 1)) == 0 && s->num_slots < INT32_MAX && (s->q_stride * 2) % 16 == 0 &&
         (s->out_stride * 2) % 16 == 0;
}

// The CTA-pair form shares 256-row items between two SMs (D = 128). Only on
// request: it measured slower than the single-CTA form on long prompts (both
// issue one N = 128 MMA per ~95 cycles, and a pair spends two SMs on one
// issuing thread).
bool prefill_pair_eligible(const ir_prefill_shape* s) {
  return prefill_tc_eligible(s) && s->head_dim == 128;
}

int prefill_path(const ir_prefill_shape* s) {
  if (g_prefill_path == 1) return 1;
  if (g_prefill_path == 2) return prefill_tc_eligible(s) ? 2 : -1;
  if (g_prefill_path == 3) return prefill_pair_eligible(s) ? 3 : -1;
  return prefill_tc_eligible(s) ? 2 : 1;
}

// Workspace of the rows-as-decode path: per-row tables and contexts, then
// the decode workspace of a batch of total_q rows.
ir_decode_shape rows_shape(const ir_prefill_shape* s) {
  ir_decode_shape d{};
  d.batch = s->total_q;
  d.num_heads = s->num_heads;
  d.num_kv_heads = s->num_kv_heads;
  d.head_dim = s->head_dim;
  d.block_size = s->block_size;
  d.max_blocks = s->max_blocks;
  d.bt_stride = s->max_blocks;
  d.q_stride = s->q_stride;
  d.out_stride = s->out_stride;
  d.num_slots = s->num_slots;
  d.scale = s->scale;
  d.dtype = s->dtype;
  return d;
}

int prefill_rows_bytes(const ir_prefill_shape* s, size_t* tables, size_t* ctx, size_t* total) {
  ir_decode_shape d = rows_shape(s);
  Plan plan;
  int rc = make_plan(&d, &plan);
  if (rc) return rc;
  *tables = align256(static_cast<size_t>(s->total_q) * s->max_blocks * 4);
  *ctx = align256(static_cast<size_t>(s->total_q) * 4);
  *total = *tables + *ctx + plan.bytes;
  return IR_OK;
}

// Scratch of ir_paged_decode_noalloc: part of the library image, so the
// entry point allocates nothing. Host code must not pass the symbol itself
// to a kernel (on the host it names a host-side shadow, not device memory);
// it passes the device address found with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_ws[IR_NOALLOC_WORKSPACE_BYTES];

std::mutex g_noalloc_mu;
// device -> (id of the context the address was found in, address of g_noalloc_ws)
std::map<int, std::pair<unsigned long long, void*>> g_noalloc_ptr;

PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;

// Unique id of the calling thread's current context (0 if none or unknown).
// A device reset ends the context; the next one has a new id, and with it a
// new copy of the library's device image at a possibly different address.
unsigned long long current_context_id() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  if (!g_ctx_current || !g_ctx_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_noalloc_ws on the current device, looked up with that
// device current on its first use and again whenever the device's context
// has changed since (after a device reset), so a stale address is never used.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(static_cast<int>(e), "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  const unsigned long long ctx = current_context_id();
  auto it = g_noalloc_ptr.find(dev);
  if (it != g_noalloc_ptr.end() && ctx != 0 && it->second.first == ctx) {
    *out = it->second.second;
    return IR_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_ws);
  if (e != cudaSuccess || p == nullptr)
    return cuda_status(e != cudaSuccess ? static_cast<int>(e) : 1,
                       "cudaGetSymbolAddress(no-alloc scratch)");
  // the lookup makes the primary context current if no context was
  g_noalloc_ptr[dev] = {ctx != 0 ? ctx : current_context_id(), p};
  *out = p;
  return IR_OK;
}

}  // namespace

namespace {

// Kernel arguments of the peer exchange from the C ABI's arrays. rows is
// batch * heads in 64 bits; it must fit the row capacity of the buffers
// (their size, which every rank allocates alike).
int peer_args(void* const* bufs, size_t buffer_bytes, int world, int rank, int64_t rows,
              int head_dim, int32_t* err, irb::PeerArgs* a) {
  if (!bufs || world <= 0 || world > 8 || rank < 0 || rank >= world)
    return fail(IR_ERR_INVALID_ARG, "world must be 1..8 and rank < world");
  if (head_dim <= 0 || head_dim > 128 || head_dim % 4 != 0 || rows < 0)
    return fail(IR_ERR_INVALID_ARG, "head_dim must be a multiple of 4 up to 128");
  const int64_t cap = irb::peer_exchange_capacity(buffer_bytes, world, head_dim);
  if (cap > INT32_MAX)
    return fail(IR_ERR_INVALID_ARG, "exchange buffer larger than 2^31 rows");
  if (rows > cap)
    return fail(IR_ERR_INVALID_ARG,
                "batch * num_heads = " + std::to_string(rows) + " rows exceed the " +
                    std::to_string(cap) + " rows an exchange buffer of " +
                    std::to_string(buffer_bytes) + " bytes holds (ir_peer_exchange_bytes)");
  *a = irb::PeerArgs{};
  for (int i = 0; i < world; ++i) {
    if (!bufs[i] || !aligned(bufs[i], 256)) return fail(IR_ERR_INVALID_ARG, "bad peer buffer");
    a->bufs[i] = static_cast<uint8_t*>(bufs[i]);
  }
  int sms = 1;
  const int e = cached(-1, sm_count_now, 0, &sms);
  if (e) return cuda_status(e, "SM count");
  a->world = world;
  a->rank = rank;
  a->rows = static_cast<int>(rows);
  a->D = head_dim;
  a->cap = static_cast<int>(cap);
  a->sms = sms;
  a->err = err;
  return IR_OK;
}
}  // namespace

extern "C" {

int ir_version(void) { return 100; }

const char* ir_last_error(void) { return g_last_error.c_str(); }

const char* ir_deverr_name(int bit) {
  static const char* names[] = {"BLOCK_ID", "CONTEXT_LEN", "SLOT",
                                "NOT_BLOCKED", "MASK", "TIMEOUT", "WRITE_SLOT"};
  if (bit < 0 || bit >= static_cast<int>(sizeof(names) / sizeof(names[0])))
    return "";
  return names[bit];
}

int ir_set_decode_path(int path) {
  if (path < 0 || path > 3) return fail(IR_ERR_INVALID_ARG, "path must be 0, 1, 2 or 3");
  std::lock_guard<std::mutex> lk(g_mu);
  g_forced_path = path == 3 ? 2 : path;
  g_one_box = path == 3 ? 0 : 1;
  return IR_OK;
}

int ir_debug_stall_next_decode(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_stall_next = 1;
  return IR_OK;
}

int ir_paged_decode_plan(const ir_decode_shape* shape, int* path,
                         int* ctas_per_kv_head) {
  Plan p;
  int rc = make_plan(shape, &p);
  if (rc) return rc;
  if (path) *path = p.path;
  if (ctas_per_kv_head) *ctas_per_kv_head = p.G;
  return IR_OK;
}

size_t ir_paged_decode_workspace_size(const ir_decode_shape* shape) {
  Plan p;
  if (make_plan(shape, &p)) return 0;
  return p.bytes;
}

int ir_cache_write(const void* k, const void* v, int64_t k_stride,
                   int64_t v_stride, void* k_pool, void* v_pool,
                   const int64_t* slot_mapping, int64_t num_tokens,
                   int num_kv_heads, int head_dim, int64_t num_slots,
                   int dtype, int32_t* err_flag, ir_stream_t stream) {
  const int eb = elem_bytes(dtype);
  if (eb == 0) return fail(IR_ERR_INVALID_ARG, "bad dtype");
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots < 0)
    return fail(IR_ERR_INVALID_ARG, "bad sizes");
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row > INT32_MAX) return fail(IR_ERR_UNSUPPORTED, "row too long");
  if (num_tokens == 0) return IR_OK;
  if (k_stride < row || v_stride < row)
    return fail(IR_ERR_INVALID_ARG, "token stride < Hkv*D");
  if (!k || !v || !k_pool || !v_pool || !slot_mapping)
    return fail(IR_ERR_INVALID_ARG, "null pointer");
  int e = irb::launch_cache_write(k, v, k_stride, v_stride, k_pool, v_pool,
                                  slot_mapping, num_tokens,
                                  static_cast<int>(row), num_slots, eb,
                                  err_flag, stream);
  return cuda_status(e, "cache write launch");
}

int ir_cache_gather(void* out, const void* pool, const int64_t* slots,
                    int64_t num_rows, int num_kv_heads, int head_dim,
                    int64_t num_slots, int dtype, int32_t* err_flag,
                    ir_stream_t stream) {
  const int eb = elem_bytes(dtype);
  if (eb == 0) return fail(IR_ERR_INVALID_ARG, "bad dtype");
  if (num_rows < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots < 0)
    return fail(IR_ERR_INVALID_ARG, "bad sizes");
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  if (row > INT32_MAX) return fail(IR_ERR_UNSUPPORTED, "row too long");
  if (num_rows == 0) return IR_OK;
  if (!out || !pool || !slots) return fail(IR_ERR_INVALID_ARG, "null pointer");
  int e = irb::launch_cache_gather(out, pool, slots, num_rows,
                                   static_cast<int>(row), num_slots, eb,
                                   err_flag, stream);
  return cuda_status(e, "cache gather launch");
}

int ir_build_decode_inputs(const int32_t* block_tables, int64_t bt_stride,
                           const int32_t* num_cached, const int64_t* last_tokens,
                           int batch, int bucket, int64_t t_max, int block_size,
                           int64_t* ids, int64_t* positions, int64_t* write_slots,
                           int64_t* gather_slots, void* mask, int mask_dtype,
                           ir_stream_t stream) {
  const int eb = elem_bytes(mask_dtype);
  if (eb == 0) return fail(IR_ERR_INVALID_ARG, "bad mask dtype");
  if (batch <= 0 || batch > bucket)
    return fail(IR_ERR_INVALID_ARG, "need 0 < batch <= bucket");
  if (t_max <= 0 || block_size <= 0 || bt_stride <= 0)
    return fail(IR_ERR_INVALID_ARG, "bad sizes");
  if (bucket > 2147483647 || (t_max + 255) / 256 > 65535)
    return fail(IR_ERR_UNSUPPORTED, "grid too large");
  if (!block_tables || !num_cached || !last_tokens || !ids || !positions || !write_slots ||
      !gather_slots || !mask)
    return fail(IR_ERR_INVALID_ARG, "null pointer");
  // finfo(dtype).min bit patterns: fp32 -3.4028235e38, bf16 -3.3895e38, fp16 -65504
  const uint32_t min_bits = mask_dtype == IR_DTYPE_F32    ? 0xff7fffffu
                            : mask_dtype == IR_DTYPE_BF16 ? 0xff7fu
                                                          : 0xfbffu;
  int e = irb::launch_build_decode_inputs(block_tables, bt_stride, num_cached, last_tokens,
                                          batch, bucket, t_max, block_size, ids, positions,
                                          write_slots, gather_slots, mask, eb, min_bits,
                                          stream);
  return cuda_status(e, "decode-inputs launch");
}

int ir_derive_block_metadata(const int64_t* gather_slots, int64_t gs_stride,
                             const void* mask, int64_t mask_stride,
                             int mask_dtype, int batch, int64_t t,
                             int block_size, int32_t* block_tables,
                             int64_t bt_stride, int32_t* context_lens,
                             int32_t* err_flag, ir_stream_t stream) {
  const int eb = elem_bytes(mask_dtype);
  if (eb == 0) return fail(IR_ERR_INVALID_ARG, "bad mask dtype");
  if (batch < 0 || t < 0 || block_size <= 0)
    return fail(IR_ERR_INVALID_ARG, "bad sizes");
  if (t > INT32_MAX) return fail(IR_ERR_UNSUPPORTED, "T overflows int32");
  if (batch == 0) return IR_OK;
  if (bt_stride < (t + block_size - 1) / block_size || gs_stride < t ||
      mask_stride < t)
    return fail(IR_ERR_INVALID_ARG, "stride smaller than row length");
  if (!gather_slots || !mask || !block_tables || !context_lens)
    return fail(IR_ERR_INVALID_ARG, "null pointer");
  int e = irb::launch_derive_metadata(gather_slots, gs_stride, mask,
                                      mask_stride, eb, batch, t, block_size,
                                      block_tables, bt_stride, context_lens,
                                      err_flag, stream);
  return cuda_status(e, "metadata launch");
}

int ir_derive_varlen_metadata(const int64_t* gather_slots, int64_t num_keys, const void* mask,
                              int64_t mask_stride, int mask_dtype, int num_rows,
                              int block_size, int max_blocks, int32_t* block_tables,
                              int32_t* context_lens, int32_t* q_start, int32_t* num_seqs,
                              int32_t* scratch, int32_t* err_flag, ir_stream_t stream) {
  const int eb = elem_bytes(mask_dtype);
  if (eb == 0) return fail(IR_ERR_INVALID_ARG, "bad mask dtype");
  if (num_rows < 0 || num_keys < 0 || block_size <= 0 || max_blocks < 0)
    return fail(IR_ERR_INVALID_ARG, "bad sizes");
  if (num_keys > INT32_MAX) return fail(IR_ERR_UNSUPPORTED, "num_keys overflows int32");
  if (mask_stride < num_keys) return fail(IR_ERR_INVALID_ARG, "mask_stride < num_keys");
  if (!q_start || !num_seqs || (num_rows > 0 && (!gather_slots || !mask || !block_tables ||
                                                 !context_lens || !scratch)))
    return fail(IR_ERR_INVALID_ARG, "null pointer");
  int e = irb::launch_derive_varlen(gather_slots, mask, mask_stride, eb, num_rows, num_keys,
                                    block_size, max_blocks, block_tables, context_lens,
                                    q_start, num_seqs, scratch, err_flag,
                                    static_cast<cudaStream_t>(stream));
  return cuda_status(e, "varlen metadata launch");
}

int ir_paged_decode(void* out, const void* q, const void* k_pool,
                    const void* v_pool, const int32_t* block_tables,
                    const int32_t* context_lens, const ir_decode_shape* shape,
                    void* workspace, size_t workspace_bytes,
                    int32_t* err_flag, ir_stream_t stream) {
  return decode_impl(Mode::kFinal, out, nullptr, nullptr, q, k_pool, v_pool,
                     nullptr, nullptr, 0, nullptr, block_tables, context_lens,
                     shape, workspace, workspace_bytes, err_flag, stream);
}

int ir_paged_decode_write(void* out, const void* q, void* k_pool, void* v_pool,
                          const void* k_new, const void* v_new,
                          int64_t kv_stride, const int64_t* slot_mapping,
                          const int32_t* block_tables,
                          const int32_t* context_lens,
                          const ir_decode_shape* shape, void* workspace,
                          size_t workspace_bytes, int32_t* err_flag,
                          ir_stream_t stream) {
  return decode_impl(Mode::kWrite, out, nullptr, nullptr, q, k_pool, v_pool,
                     k_new, v_new, kv_stride, slot_mapping, block_tables,
                     context_lens, shape, workspace, workspace_bytes, err_flag,
                     stream);
}

int ir_paged_decode_rope_write(void* out, const void* q, void* k_pool, void* v_pool,
                               const void* k_new, const void* v_new,
                               int64_t kv_stride, const int64_t* slot_mapping,
                               const float* rope_cos, const float* rope_sin,
                               int64_t rope_stride, const int32_t* block_tables,
                               const int32_t* context_lens,
                               const ir_decode_shape* shape, void* workspace,
                               size_t workspace_bytes, int32_t* err_flag,
                               ir_stream_t stream) {
  if (!rope_cos || !rope_sin) return fail(IR_ERR_INVALID_ARG, "null rope_cos / rope_sin");
  return decode_impl(Mode::kWrite, out, nullptr, nullptr, q, k_pool, v_pool,
                     k_new, v_new, kv_stride, slot_mapping, block_tables,
                     context_lens, shape, workspace, workspace_bytes, err_flag,
                     stream, rope_cos, rope_sin, rope_stride);
}

int ir_paged_decode_rope(void* out, const void* q, const void* k_pool, const void* v_pool,
                         const float* rope_cos, const float* rope_sin, int64_t rope_stride,
                         const int32_t* block_tables, const int32_t* context_lens,
                         const ir_decode_shape* shape, void* workspace,
                         size_t workspace_bytes, int32_t* err_flag, ir_stream_t stream) {
  if (!rope_cos || !rope_sin) return fail(IR_ERR_INVALID_ARG, "null rope_cos / rope_sin");
  return decode_impl(Mode::kFinal, out, nullptr, nullptr, q, k_pool, v_pool, nullptr,
                     nullptr, 0, nullptr, block_tables, context_lens, shape, workspace,
                     workspace_bytes, err_flag, stream, rope_cos, rope_sin, rope_stride);
}

int ir_kv_proj_rope_write(const void* x, int64_t x_stride, int num_tokens, int hidden,
                          const void* w_k, const void* w_v, const void* b_k,
                          const void* b_v, const float* rope_cos, const float* rope_sin,
                          int64_t rope_stride, const int64_t* slot_mapping, void* k_pool,
                          void* v_pool, int64_t num_slots, int num_kv_heads, int head_dim,
                          int dtype, int32_t* err_flag, ir_stream_t stream) {
  if (dtype != IR_DTYPE_BF16 && dtype != IR_DTYPE_F16)
    return fail(IR_ERR_UNSUPPORTED, "the projection kernel takes bf16 or fp16");
  if (head_dim != 64 && head_dim != 128)
    return fail(IR_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (num_tokens < 0 || num_kv_heads <= 0 || num_kv_heads > 256)
    return fail(IR_ERR_INVALID_ARG, "bad num_tokens / num_kv_heads");
  if (hidden < 64 || hidden % 64 != 0)
    return fail(IR_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  if (num_tokens == 0) return IR_OK;
  if (!x || !w_k || !w_v || !slot_mapping || !k_pool || !v_pool)
    return fail(IR_ERR_INVALID_ARG, "null pointer");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return fail(IR_ERR_INVALID_ARG, "rope_cos and rope_sin must both be given");
  if (rope_cos && (rope_stride < head_dim || !aligned(rope_cos, 4) || !aligned(rope_sin, 4)))
    return fail(IR_ERR_INVALID_ARG, "rope tables: stride < head_dim or not 4-byte aligned");
  if (x_stride < hidden || (x_stride * 2) % 16 != 0 || !aligned(x, 16) || !aligned(w_k, 16) ||
      !aligned(w_v, 16))
    return fail(IR_ERR_INVALID_ARG,
                "x, w_k, w_v must be 16-byte aligned with 16-byte row strides");
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || num_slots <= 0)
    return fail(IR_ERR_INVALID_ARG, "pools must be 16-byte aligned and non-empty");
  const int64_t n_out = static_cast<int64_t>(num_kv_heads) * head_dim;
  CUtensorMap tmx, tmwk, tmwv;
  if (!make_rows_map(&tmx, x, num_tokens, hidden, x_stride, dtype, 128) ||
      !make_rows_map(&tmwk, w_k, n_out, hidden, hidden, dtype, head_dim) ||
      !make_rows_map(&tmwv, w_v, n_out, hidden, hidden, dtype, head_dim))
    return fail(IR_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  irb::KvProjArgs a{};
  a.M = num_tokens;
  a.K = hidden;
  a.Hkv = num_kv_heads;
  a.D = head_dim;
  a.bias_k = b_k;
  a.bias_v = b_v;
  a.cos = rope_cos;
  a.sin = rope_sin;
  a.rope_stride = rope_stride;
  a.slots = slot_mapping;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_slots = num_slots;
  a.err = err_flag;
  return cuda_status(irb::launch_kv_proj(tmx, tmwk, tmwv, a, dtype,
                                         static_cast<cudaStream_t>(stream)),
                     "K/V projection launch");
}

int ir_paged_decode_lse(float* o, float* lse, const void* q,
                        const void* k_pool, const void* v_pool,
                        const int32_t* block_tables,
                        const int32_t* context_lens,
                        const ir_decode_shape* shape, void* workspace,
                        size_t workspace_bytes, int32_t* err_flag,
                        ir_stream_t stream) {
  return decode_impl(Mode::kLse, nullptr, o, lse, q, k_pool, v_pool, nullptr,
                     nullptr, 0, nullptr, block_tables, context_lens, shape,
                     workspace, workspace_bytes, err_flag, stream);
}

int ir_paged_decode_noalloc(void* out, const void* q, const void* k_pool,
                            const void* v_pool, const int32_t* block_tables,
                            const int32_t* context_lens,
                            const ir_decode_shape* shape_in, int32_t* err_flag,
                            ir_stream_t stream) {
  if (!shape_in) return fail(IR_ERR_INVALID_ARG, "shape is null");
  ir_decode_shape local = *shape_in;  // the built-in scratch keeps the static schedule
  local.flags = 0;
  const ir_decode_shape* shape = &local;
  Plan plan;
  int rc = make_plan(shape, &plan);
  if (rc) return rc;
  if (plan.bytes > IR_NOALLOC_WORKSPACE_BYTES)
    return fail(IR_ERR_WORKSPACE,
                "shape needs " + std::to_string(plan.bytes) +
                    " bytes of scratch; ir_paged_decode_noalloc holds at most " +
                    std::to_string(IR_NOALLOC_WORKSPACE_BYTES) +
                    " (use ir_paged_decode with a caller workspace)");
  void* ws = nullptr;
  rc = noalloc_scratch(&ws);
  if (rc) return rc;
  return decode_impl(Mode::kFinal, out, nullptr, nullptr, q, k_pool, v_pool,
                     nullptr, nullptr, 0, nullptr, block_tables, context_lens,
                     shape, ws, IR_NOALLOC_WORKSPACE_BYTES, err_flag, stream);
}

int ir_lse_merge(void* out, int64_t out_stride, const float* o_parts,
                 int64_t o_part_stride, const float* lse_parts,
                 int64_t lse_part_stride, int num_parts, int batch,
                 int num_heads, int head_dim, int dtype, ir_stream_t stream) {
  if (elem_bytes(dtype) == 0) return fail(IR_ERR_INVALID_ARG, "bad dtype");
  if (num_parts <= 0 || batch < 0 || num_heads <= 0 || head_dim <= 0)
    return fail(IR_ERR_INVALID_ARG, "bad sizes");
  if (batch == 0) return IR_OK;
  const int64_t rows = static_cast<int64_t>(batch) * num_heads;
  if (out_stride < static_cast<int64_t>(num_heads) * head_dim)
    return fail(IR_ERR_INVALID_ARG, "out_stride < H*D");
  if (num_parts > 1 && (o_part_stride < rows * head_dim || lse_part_stride < rows))
    return fail(IR_ERR_INVALID_ARG, "part strides smaller than one part");
  if (!out || !o_parts || !lse_parts) return fail(IR_ERR_INVALID_ARG, "null pointer");
  if (batch > 2147483647 || num_heads > 65535)
    return fail(IR_ERR_UNSUPPORTED, "grid too large");
  int e = irb::launch_lse_merge(out, out_stride, o_parts, o_part_stride, lse_parts,
                                lse_part_stride, num_parts, batch, num_heads, head_dim,
                                dtype, stream);
  return cuda_status(e, "lse merge launch");
}

int ir_set_prefill_path(int path) {
  if (path < 0 || path > 3) return fail(IR_ERR_INVALID_ARG, "path must be 0, 1, 2 or 3");
  std::lock_guard<std::mutex> lk(g_mu);
  g_prefill_path = path;
  return IR_OK;
}

int ir_paged_prefill_plan(const ir_prefill_shape* shape, int* path) {
  int rc = check_prefill_shape(shape);
  if (rc) return rc;
  const int p = prefill_path(shape);
  if (p < 0) return fail(IR_ERR_UNSUPPORTED, "tensor-core prefill forced but shape not eligible");
  if (path) *path = p;
  return IR_OK;
}

size_t ir_paged_prefill_workspace_size(const ir_prefill_shape* shape) {
  if (check_prefill_shape(shape)) return 0;
  if (prefill_path(shape) != 1) return 0;
  size_t t, c, total;
  if (prefill_rows_bytes(shape, &t, &c, &total)) return 0;
  return total;
}

int ir_paged_prefill(void* out, const void* q, const void* k_pool, const void* v_pool,
                     const int32_t* block_tables, const int32_t* context_lens,
                     const int32_t* q_start, const ir_prefill_shape* s, void* workspace,
                     size_t workspace_bytes, int32_t* err_flag, ir_stream_t stream) {
  int rc = check_prefill_shape(s);
  if (rc) return rc;
  if (s->num_seqs == 0 || s->total_q == 0) return IR_OK;
  if (!out || !q || !k_pool || !v_pool || !context_lens || !q_start ||
      (s->max_blocks > 0 && !block_tables))
    return fail(IR_ERR_INVALID_ARG, "null pointer");
  int path = prefill_path(s);
  if (path < 0) return fail(IR_ERR_UNSUPPORTED, "tensor-core prefill forced but shape not eligible");
  if (path >= 2 && !(aligned(q, 16) && aligned(out, 16) && aligned(k_pool, 16) &&
                     aligned(v_pool, 16))) {
    if (g_prefill_path >= 2)
      return fail(IR_ERR_UNSUPPORTED, "tensor-core prefill forced but pointers misaligned");
    path = 1;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (path >= 2) {
    const bool pair = path == 3;
    irb::PrefillArgs a{};
    a.q = q;
    a.q_stride = s->q_stride;
    a.out = out;
    a.out_stride = s->out_stride;
    a.block_tables = block_tables;
    a.bt_stride = s->bt_stride;
    a.context_lens = context_lens;
    a.q_start = q_start;
    a.S = s->num_seqs;
    a.total_q = s->total_q;
    a.H = s->num_heads;
    a.Hkv = s->num_kv_heads;
    a.n_rep = s->num_heads / s->num_kv_heads;
    a.D = s->head_dim;
    a.bs = s->block_size;
    a.max_blocks = s->max_blocks;
    a.num_slots = s->num_slots;
    a.num_blocks = s->num_slots / s->block_size;
    a.scale_log2 = s->scale * irb::kLog2e;
    a.err = err_flag;
    CUtensorMap tmq, tmk, tmv;
    const int rows = s->block_size < 128 ? s->block_size : 128;
    // a CTA of a pair stages 64 keys of each K tile
    const int krows = pair && rows > 64 ? 64 : rows;
    if (!make_q_map(&tmq, q, s->total_q, s->num_heads, s->head_dim, s->q_stride, s->dtype) ||
        !make_pool_map(&tmk, k_pool, s->num_slots, s->num_kv_heads, s->head_dim, s->dtype,
                       krows) ||
        !make_pool_map(&tmv, v_pool, s->num_slots, s->num_kv_heads, s->head_dim, s->dtype,
                       rows))
      return fail(IR_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    int sms = 0;
    int rc2 = cached(-1, sm_count_now, 0, &sms);
    if (rc2) return cuda_status(rc2, "device query");
    int e = irb::launch_prefill_tc(tmq, tmk, tmv, a, s->dtype, sms > 0 ? sms : 148, pair, st);
    return cuda_status(e, "prefill kernel launch");
  }
  // rows as decode rows: each query row is a sequence of context position + 1
  size_t tb, cb, total;
  rc = prefill_rows_bytes(s, &tb, &cb, &total);
  if (rc) return rc;
  if (!workspace || workspace_bytes < total)
    return fail(IR_ERR_WORKSPACE, "workspace smaller than ir_paged_prefill_workspace_size");
  if (!aligned(workspace, 256)) return fail(IR_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int32_t* row_bt = reinterpret_cast<int32_t*>(ws);
  int32_t* row_ctx = reinterpret_cast<int32_t*>(ws + tb);
  int e = irb::launch_prefill_rows(block_tables, s->bt_stride, context_lens, q_start, s->num_seqs,
                                   s->total_q, s->max_blocks, s->max_blocks * s->block_size,
                                   row_bt, row_ctx, err_flag, st);
  if (e) return cuda_status(e, "prefill row tables");
  ir_decode_shape d = rows_shape(s);
  return decode_impl(Mode::kFinal, out, nullptr, nullptr, q, k_pool, v_pool, nullptr, nullptr, 0,
                     nullptr, row_bt, row_ctx, &d, ws + tb + cb, workspace_bytes - tb - cb,
                     err_flag, st);
}

// ---------------------------------------------------------------- peer exchange

int ir_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(IR_ERR_INVALID_ARG, "null pointer or zero size");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  return cuda_status(static_cast<int>(e), "peer buffer allocation");
}

int ir_peer_free(void* ptr) { return cuda_status(static_cast<int>(cudaFree(ptr)), "cudaFree"); }

int ir_peer_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return fail(IR_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e == cudaSuccess) std::memcpy(handle, &h, sizeof(h));
  return cuda_status(static_cast<int>(e), "cudaIpcGetMemHandle");
}

int ir_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(IR_ERR_INVALID_ARG, "null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cuda_status(
      static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess)),
      "cudaIpcOpenMemHandle");
}

int ir_peer_close(void* ptr) {
  return cuda_status(static_cast<int>(cudaIpcCloseMemHandle(ptr)), "cudaIpcCloseMemHandle");
}

size_t ir_peer_exchange_bytes(int world, int rows, int head_dim) {
  if (world <= 0 || world > 8 || rows < 0 || head_dim <= 0) return 0;
  return irb::peer_exchange_bytes(world, rows, head_dim);
}

int ir_peer_exchange(void* out, int64_t out_stride, const float* o, const float* lse,
                     void* const* bufs, size_t buffer_bytes, int world, int rank, int batch,
                     int num_heads, int head_dim, int dtype, int32_t* err_flag,
                     ir_stream_t stream) {
  irb::PeerArgs a;
  if (batch < 0 || num_heads <= 0) return fail(IR_ERR_INVALID_ARG, "bad batch / num_heads");
  int rc = peer_args(bufs, buffer_bytes, world, rank,
                     static_cast<int64_t>(batch) * num_heads, head_dim, err_flag, &a);
  if (rc) return rc;
  if (!o || !lse || !aligned(o, 16)) return fail(IR_ERR_INVALID_ARG, "o must be 16-byte aligned");
  if (!out || elem_bytes(dtype) == 0 || out_stride < static_cast<int64_t>(num_heads) * head_dim)
    return fail(IR_ERR_INVALID_ARG, "bad output");
  return cuda_status(irb::launch_peer_exchange(out, out_stride, o, lse, num_heads, dtype, a,
                                               static_cast<cudaStream_t>(stream)),
                     "peer exchange launch");
}

}  // extern "C"
