// Log-sum-exp combine of per-chunk partials (m, l, acc) into O.
//
// One warp per output row (b, head, position): M = max_s m_s,
// w_s = exp2(m_s - M), O = sum_s w_s acc_s / sum_s w_s l_s.
// Reference: gqa_split_reduce_kernel, gqa_kernels/gqa_split.py:115-147
// (body :134-147). The same kernel serves the cross-GPU combine, where the
// split index runs over ranks instead of key chunks.
#pragma once

#include "gqa_common.cuh"

namespace gqa {

struct CombineParams {
  const float* m;
  const float* l;
  const float* acc;
  void* o;
  int64_t p_sb, p_sh, p_sm, p_ss;          // strides of m / l (elements)
  int64_t a_sb, a_sh, a_sm, a_ss, a_sd;    // strides of acc
  int64_t o_sb, o_sh, o_sm;                // strides of O (d stride 1)
  int batch, hq, seq_q, head_dim, nsplit;
  // Peer exchange (cnt != nullptr): the parts are the ranks' slots in this rank's
  // receive buffer, written by the ranks' partial kernels over NVLink. The kernel
  // first waits (bounded) until every source's counter reaches epoch x units (each
  // source adds one per unit after that unit's rows), then reads the parity
  // (epoch & 1) half, parity_stride floats from the first.
  const unsigned long long* cnt;
  const unsigned long long* epoch;
  unsigned long long units;
  int64_t parity_stride;
};

template <bool BF16>
__global__ void __launch_bounds__(128) gqa_combine_kernel(const CombineParams p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int64_t parity_off = 0;
  if (p.cnt) {
    // Bounded wait for every source's rows: thread 0 acquires (system scope) each
    // counter; the CTA barrier orders the other threads' reads after it. A source
    // that never arrives leaves GQA_ERR_TIMEOUT in the device error word and O as it
    // was.
    __shared__ int arrived;
    const unsigned long long e = *p.epoch;
    if (threadIdx.x == 0) {
      const unsigned long long target = e * p.units;
      const uint64_t t0 = globaltimer_ns();
      int ok = 1;
      for (int s = 0; s < p.nsplit && ok; ++s) {
        while (ld_acquire_sys_u64(p.cnt + s) < target) {
          if (globaltimer_ns() - t0 > wait_limit_ns()) {
            report_device_error(GQA_ERR_TIMEOUT, 301);
            ok = 0;
            break;
          }
          __nanosleep(32);
        }
      }
      arrived = ok;
    }
    __syncthreads();
    if (!arrived) return;
    parity_off = (int64_t)(e & 1ull) * p.parity_stride;
  }
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  const int64_t n_rows = (int64_t)p.batch * p.hq * p.seq_q;
  if (row >= n_rows) return;
  const int pos = (int)(row % p.seq_q);
  const int head = (int)((row / p.seq_q) % p.hq);
  const int b = (int)(row / ((int64_t)p.seq_q * p.hq));
  // Reads through L2 (.cg): the parts may have been written by other GPUs.
  const float* mrow = p.m + parity_off + b * p.p_sb + head * p.p_sh + (int64_t)pos * p.p_sm;
  const float* lrow = p.l + parity_off + b * p.p_sb + head * p.p_sh + (int64_t)pos * p.p_sm;
  const float* arow = p.acc + parity_off + b * p.a_sb + head * p.a_sh + (int64_t)pos * p.a_sm;

  float M = -INFINITY;
  for (int s = lane; s < p.nsplit; s += 32) M = fmaxf(M, __ldcg(mrow + s * p.p_ss));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  // All-empty rows (M = -inf) give weights 0 and L = 0, so O = 0/0 = NaN as in the reference.
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
  for (int s = lane; s < p.nsplit; s += 32) L += fast_exp2(__ldcg(mrow + s * p.p_ss) - Mu) * __ldcg(lrow + s * p.p_ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
  const float inv = 1.f / L;

  uint16_t* orow = reinterpret_cast<uint16_t*>(p.o) + b * p.o_sb + head * p.o_sh + (int64_t)pos * p.o_sm;
  for (int d = lane * 2; d < p.head_dim; d += 64) {
    float a0 = 0.f, a1 = 0.f;
    for (int s = 0; s < p.nsplit; ++s) {
      const float w = fast_exp2(__ldcg(mrow + s * p.p_ss) - Mu);
      a0 += w * __ldcg(arow + s * p.a_ss + d * p.a_sd);
      a1 += w * __ldcg(arow + s * p.a_ss + (d + 1) * p.a_sd);
    }
    *reinterpret_cast<uint32_t*>(orow + d) = pack2<BF16>(a0 * inv, a1 * inv);
  }
}

// One step of a peer exchange's call counter (one thread; stream-ordered before the
// call's partial and combine kernels, which read it).
__global__ void gqa_epoch_bump_kernel(unsigned long long* epoch) { *epoch += 1ull; }

// O[...] = NaN for every element (seq_kv == 0: no key is visible to any row,
// the reference's 0/0).
__global__ void gqa_fill_nan_kernel(uint16_t* o, int64_t o_sb, int64_t o_sh, int64_t o_sm, int batch, int hq,
                                    int seq_q, int head_dim, uint16_t nan_bits) {
  const int64_t n = (int64_t)batch * hq * seq_q * head_dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % head_dim);
    const int64_t r = i / head_dim;
    const int pos = (int)(r % seq_q);
    const int head = (int)((r / seq_q) % hq);
    const int b = (int)(r / ((int64_t)seq_q * hq));
    o[b * o_sb + head * o_sh + (int64_t)pos * o_sm + d] = nan_bits;
  }
}

// The partial of an empty key range: m = -inf, l = 0, acc = 0 for every row (rows
// m/l, rows x head_dim acc, contiguous). A rank whose key shard holds no key
// contributes it; the combine gives it weight exp2(-inf - M) = 0.
__global__ void gqa_fill_empty_partial_kernel(float* m, float* l, float* acc, int64_t rows, int head_dim) {
  const int64_t n = rows * head_dim;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    acc[i] = 0.f;
    if (i < rows) {
      m[i] = -INFINITY;
      l[i] = 0.f;
    }
  }
}

}  // namespace gqa
