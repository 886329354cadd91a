// Cache write of the vLLM-shaped paged interface: each new token's K and V rows are
// scattered into the paged caches through a slot mapping (slot = block * block_size +
// position in the block; a negative slot marks a padding token, which is skipped).
// 16-bit caches get the rows as they are; e4m3 caches get x / scale rounded to nearest
// even and saturated to +-448 (vLLM's fp8 KV-cache convention: real value = stored
// value x scale).
//
// Byte work, bound by HBM (or by latency, for one decode token per sequence): one warp
// moves one (token, kv head) row with coalesced 8-byte (head_dim 128) or 4-byte
// (head_dim 64) accesses per lane. A slot past the cache is never written: the row is
// skipped and GQA_ERR_INVALID_ARG is recorded in the device error word (site 201).
#pragma once

#include "gqa_common.cuh"

namespace gqa {

struct AppendParams {
  const uint16_t* key;
  const uint16_t* value;
  int64_t k_st, k_sh;  // element strides of key (token, kv head); the d stride is 1
  int64_t v_st, v_sh;
  void* k_cache;       // (num_blocks, block_size, hkv, head_dim), contiguous
  void* v_cache;
  const int64_t* slot_mapping;  // (num_tokens,)
  int num_tokens, hkv;
  int64_t num_slots;  // num_blocks * block_size
  float k_scale, v_scale;
};

// Two floats to two e4m3 bytes (lo -> low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <bool BF16>
__device__ __forceinline__ float2 to_f32x2(uint32_t x) {
  if constexpr (BF16) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&x));
  }
}

// One row of HD elements: EPL = HD / 32 per lane.
template <int HD, bool BF16, bool FP8>
__device__ __forceinline__ void append_row(const uint16_t* src, void* cache, int64_t dst, float scale, int lane) {
  constexpr int EPL = HD / 32;
  const int d = lane * EPL;
  if constexpr (EPL == 4) {
    const uint2 x = *reinterpret_cast<const uint2*>(src + d);
    if constexpr (FP8) {
      const float2 a = to_f32x2<BF16>(x.x), b = to_f32x2<BF16>(x.y);
      const uint32_t q = f32x2_to_e4m3x2(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale)) |
                         (f32x2_to_e4m3x2(__fdiv_rn(b.x, scale), __fdiv_rn(b.y, scale)) << 16);
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(cache) + dst + d) = q;
    } else {
      *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(cache) + dst + d) = x;
    }
  } else {
    const uint32_t x = *reinterpret_cast<const uint32_t*>(src + d);
    if constexpr (FP8) {
      const float2 a = to_f32x2<BF16>(x);
      *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(cache) + dst + d) =
          (uint16_t)f32x2_to_e4m3x2(__fdiv_rn(a.x, scale), __fdiv_rn(a.y, scale));
    } else {
      *reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(cache) + dst + d) = x;
    }
  }
}

template <int HD, bool BF16, bool FP8>
__global__ void __launch_bounds__(256) gqa_kv_append_kernel(const AppendParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)p.num_tokens * p.hkv;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int tok = (int)(r / p.hkv), h = (int)(r - (int64_t)tok * p.hkv);
    const int64_t slot = p.slot_mapping[tok];
    if (slot < 0) continue;  // padding token
    if (slot >= p.num_slots) {
      if (lane == 0) report_device_error(GQA_ERR_INVALID_ARG, 201);
      continue;
    }
    const int64_t dst = (slot * p.hkv + h) * HD;  // elements (bytes for e4m3) into the cache
    append_row<HD, BF16, FP8>(p.key + tok * p.k_st + h * p.k_sh, p.k_cache, dst, p.k_scale, lane);
    append_row<HD, BF16, FP8>(p.value + tok * p.v_st + h * p.v_sh, p.v_cache, dst, p.v_scale, lane);
  }
}

}  // namespace gqa
