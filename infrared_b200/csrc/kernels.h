// Host-side launchers of the infrared_b200 kernels (internal interface
// between the C ABI in capi.cu and the kernel translation units).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace irb {

struct DecodeArgs;

// decode_tma.cu: 16-bit pools, D in {64, 128}, group <= 8, bs == 8 or bs % 16 == 0
int launch_decode_tma(const CUtensorMap& tmk, const CUtensorMap& tmv,
                      const DecodeArgs& a, int dtype, cudaStream_t stream);
int decode_tma_occupancy(int dtype, int D, int bs);

// decode_generic.cu: any dtype, D in {64, 128}, group <= 16, any block size
int launch_decode_generic(const DecodeArgs& a, int dtype, cudaStream_t stream);
int decode_generic_occupancy(int dtype, int D);

// merges of split sequences (decode_generic.cu)
int launch_split_merge(const DecodeArgs& a, int dtype, cudaStream_t stream);
int launch_lse_merge(void* out, int64_t out_stride, const float* o_parts,
                     const float* lse_parts, int P, int B, int H, int D,
                     int dtype, cudaStream_t stream);

// cache_ops.cu
int launch_cache_write(const void* k, const void* v, int64_t k_stride,
                       int64_t v_stride, void* k_pool, void* v_pool,
                       const int64_t* slots, int64_t n, int row_elems,
                       int64_t num_slots, int elem_bytes, int32_t* err,
                       cudaStream_t stream);
int launch_cache_gather(void* out, const void* pool, const int64_t* slots,
                        int64_t n, int row_elems, int64_t num_slots,
                        int elem_bytes, int32_t* err, cudaStream_t stream);
int launch_derive_metadata(const int64_t* gs, int64_t gs_stride,
                           const void* mask, int64_t mask_stride,
                           int mask_elem_bytes, int B, int64_t T, int bs,
                           int32_t* bt, int64_t bt_stride, int32_t* ctx,
                           int32_t* err, cudaStream_t stream);

}  // namespace irb
