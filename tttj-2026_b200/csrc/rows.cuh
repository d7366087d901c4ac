// K4 row kernels and the token plan.
//
// * plan_tokens_kernel: turns valid_token_mask [B, S] into the packed valid-token
//   layout (per-sequence valid counts and offsets, packed row -> source token,
//   source token -> packed row or -1) and the attention work list ordered
//   longest-first.  Replaces the reference's host-side mask handling
//   (kernels/sequence_resident.py:164-192, kernels/case14_hybrid.py:642-672) with a
//   device-side pass, so a forward never synchronises with the host.
// * layernorm rows: nn.LayerNorm(d_model) (benchmarks/torch_transformer_benchmark.py:128,
//   130, 160): biased variance, eps 1e-5, fp32 statistics, affine.
//   - ln_gather_kernel: reads the caller's x (fp16 or fp32) at the packed rows,
//     writes the fp32 residual stream, its fp16 copy and layer 0's LN1 statistics.
//     Every other LayerNorm of the stack is folded into the GEMM that consumes it
//     (fold_ln_kernel prepares the weights once per plan).
//   - ln_rows_kernel: LN of fp16 rows (the per-kernel layernorm entry point).
//   - ln_final_scatter_kernel: final LayerNorm + masked_fill(~mask, 0)
//     (torch_transformer_benchmark.py:168-171), written back to [B, S, D] in the
//     caller's dtype.
#pragma once
#include "common.cuh"
#include "params.h"

namespace tttj {

// Number of non-zero bytes among 16 mask bytes.
__device__ __forceinline__ int mask16_count(uint4 m) {
  int c = 0;
  const uint32_t w[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // Each byte -> 1 if non-zero: fold the byte's bits into its lowest bit.
    uint32_t v = w[i];
    v |= v >> 4;
    v |= v >> 2;
    v |= v >> 1;
    c += __popc(v & 0x01010101u);
  }
  return c;
}

// Single-CTA plan.  Dynamic shared memory: (2*B + 1 + nkeys + 1) ints rounded up to 16
// bytes, then 512 bytes of mask staging per warp.  Attention items
// are listed for the query blocks starting in [q_lo, q_hi) of each sequence (a rank's
// share of a sequence split across ranks; 0 and INT_MAX otherwise).
__global__ void __launch_bounds__(PLAN_THREADS) plan_tokens_kernel(const uint8_t* __restrict__ mask,
                                                                   int B, int S, int H, int causal,
                                                                   int q_block, int kv_block,
                                                                   int q_lo, int q_hi,
                                                                   TokenPlan plan) {
  griddep_wait();
  griddep_launch();
  extern __shared__ int sh[];
  const int nkeys = (S + kv_block - 1) / kv_block + 1;
  int* cnt = sh;             // [B]
  int* off = sh + B;         // [B+1]
  int* hist = sh + 2 * B + 1;  // [nkeys+1]
  // Per-warp 512-byte mask staging slots after the ints (16-byte aligned).
  uint4* stage = reinterpret_cast<uint4*>(sh + ((2 * B + 1 + nkeys + 1 + 3) & ~3));
  const int warp = warp_id();
  const int lane = lane_id();
  const int nwarps = blockDim.x >> 5;

  for (int i = threadIdx.x; i <= nkeys; i += blockDim.x) hist[i] = 0;
  for (int i = threadIdx.x; i < PLAN_COUNTERS; i += blockDim.x) plan.counters[i] = 0;
  // Mask bytes are read 16 per lane (512 positions per warp step) when the rows are
  // 16-byte aligned, else one per lane.
  const bool vec_mask = mask != nullptr && (S % 16) == 0 &&
                        (reinterpret_cast<uintptr_t>(mask) & 15) == 0;
  for (int b = warp; b < B; b += nwarps) {
    int c = 0;
    if (mask == nullptr) {
      c = S;
    } else if (vec_mask) {
      const uint4* row = reinterpret_cast<const uint4*>(mask + (size_t)b * S);
      for (int i = lane; i < S / 16; i += 32) c += mask16_count(row[i]);
      for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffff, c, o);
    } else {
      for (int s = lane; s < S; s += 32) c += mask[(size_t)b * S + s] != 0;
      for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffff, c, o);
    }
    if (lane == 0) cnt[b] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = 0; b < B; ++b) {
      off[b] = acc;
      acc += cnt[b];
    }
    off[B] = acc;
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    plan.seq_len[b] = cnt[b];
    plan.seq_off[b] = off[b];
  }
  if (threadIdx.x == 0) plan.seq_off[B] = off[B];

  // Packed row maps: a warp per sequence, ballot scan over 32 positions at a time (so
  // every map store is one coalesced 128-byte row).  Vector path: each 512-position step
  // of the sequence's mask is first staged in this warp's shared-memory slot, 16 bytes
  // per lane, so the scan reads shared memory instead of waiting on one global load per
  // 32 positions.
  for (int b = warp; b < B && vec_mask; b += nwarps) {
    int running = off[b];
    const uint4* row = reinterpret_cast<const uint4*>(mask + (size_t)b * S);
    uint8_t* slot = reinterpret_cast<uint8_t*>(stage) + warp * 512;
    for (int s0 = 0; s0 < S; s0 += 512) {
      const int sv = s0 + 16 * lane;
      reinterpret_cast<uint4*>(slot)[lane] = sv < S ? row[sv / 16] : make_uint4(0u, 0u, 0u, 0u);
      __syncwarp();
#pragma unroll 4
      for (int k = 0; k < 16; ++k) {
        const int s = s0 + 32 * k + lane;
        const bool in = s < S;
        const bool v = in && slot[32 * k + lane] != 0;
        const unsigned bal = __ballot_sync(0xffffffff, v);
        const int rank = __popc(bal & ((1u << lane) - 1u));
        if (in) {
          const int tok = b * S + s;
          if (v) {
            plan.packed_src[running + rank] = tok;
            plan.dst_map[tok] = running + rank;
          } else {
            plan.dst_map[tok] = -1;
          }
        }
        running += __popc(bal);
      }
      __syncwarp();
    }
  }
  for (int b = warp; b < B && !vec_mask; b += nwarps) {
    int running = off[b];
    for (int s0 = 0; s0 < S; s0 += 32) {
      const int s = s0 + lane;
      const bool in = s < S;
      const bool v = in && (mask == nullptr || mask[(size_t)b * S + s] != 0);
      const unsigned bal = __ballot_sync(0xffffffff, v);
      const int rank = __popc(bal & ((1u << lane) - 1u));
      if (in) {
        const int tok = b * S + s;
        if (v) {
          plan.packed_src[running + rank] = tok;
          plan.dst_map[tok] = running + rank;
        } else {
          plan.dst_map[tok] = -1;
        }
      }
      running += __popc(bal);
    }
  }

  // Attention work list, longest first: key = number of kv blocks the item streams.
  const int qt_max = (S + q_block - 1) / q_block;
  for (int i = threadIdx.x; i < B * qt_max; i += blockDim.x) {
    const int b = i / qt_max;
    const int qt = i - b * qt_max;
    const int len = cnt[b];
    if (qt * q_block < len && qt * q_block >= q_lo && qt * q_block < q_hi) {
      const int kv_end = causal ? min(len, (qt + 1) * q_block) : len;
      const int key = (kv_end + kv_block - 1) / kv_block;
      atomicAdd(&hist[key], H);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int k = nkeys; k >= 0; --k) {
      const int c = hist[k];
      hist[k] = acc;  // start offset of bucket k (descending keys)
      acc += c;
    }
    *plan.item_count = acc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < B * qt_max; i += blockDim.x) {
    const int b = i / qt_max;
    const int qt = i - b * qt_max;
    const int len = cnt[b];
    if (qt * q_block < len && qt * q_block >= q_lo && qt * q_block < q_hi) {
      const int kv_end = causal ? min(len, (qt + 1) * q_block) : len;
      const int key = (kv_end + kv_block - 1) / kv_block;
      const int pos = atomicAdd(&hist[key], H);
      for (int h = 0; h < H; ++h) plan.items[pos + h] = make_int2(b, (qt << 8) | h);
    }
  }
}

// ---------------------------------------------------------------------------
// LayerNorm: one warp per row, each lane holds VPL 8-element vectors (D <= 256*VPL).
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__half>(const __half* src, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_half2(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <>
__device__ __forceinline__ void load8<float>(const float* src, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(src)[0];
  const float4 b = reinterpret_cast<const float4*>(src)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8(__half* dst, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(dst) = make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]),
                                              pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
}
__device__ __forceinline__ void store8(float* dst, const float (&v)[8]) {
  reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

template <int VPL>
__device__ __forceinline__ void ln_normalise(float (&x)[VPL][8], int D, const float* gamma,
                                             const float* beta, float eps) {
  const int lane = lane_id();
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if ((lane + 32 * i) * 8 < D) {
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += x[i][e];
    }
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
  const float mean = sum / (float)D;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if ((lane + 32 * i) * 8 < D) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = x[i][e] - mean;
        sq += d * d;
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffff, sq, o);
  const float rstd = rsqrtf(sq / (float)D + eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) {
      float g[8], bb[8];
      load8<float>(gamma + c, g);
      load8<float>(beta + c, bb);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[i][e] = (x[i][e] - mean) * rstd * g[e] + bb[e];
    }
  }
}

// Layer-0 entry: gather the caller's rows into the packed fp32 residual stream and
// prepare layer 0's LN1 the way the residual GEMM epilogues prepare every later
// LayerNorm: the row's exact mean (two passes over the row held in registers) is its
// pivot c, the fp16 copy (A operand of the LayerNorm-folded QKV GEMM) holds x - c, and
// partial 0 of the row's n_parts statistics partials holds the (sum, sum of squares)
// of x - c (the other partials zero).  Block 0 also zeroes the forward's attention
// work counters, so a forward that reuses the token plan (no plan kernel) starts from
// zero as well, even after an earlier launch gave up part-way.  This runs after
// griddep_wait, i.e. after every kernel of the previous forward has completed.
template <int VPL, typename TIn>
__global__ void __launch_bounds__(256) ln_gather_kernel(const TIn* __restrict__ x,
                                                        const int* __restrict__ packed_src,
                                                        const int* __restrict__ rows_dev, int D,
                                                        float* resid, __half* x16, float2* stats,
                                                        float* pivot, int n_parts, int* counters) {
  griddep_wait();
  griddep_launch();
  if (blockIdx.x == 0 && counters != nullptr)
    for (int i = threadIdx.x; i < PLAN_COUNTERS; i += blockDim.x) counters[i] = 0;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (row >= *rows_dev) return;
  const int src = packed_src[row];
  const int lane = lane_id();
  float v[VPL][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) {
      load8<TIn>(x + (size_t)src * D + c, v[i]);
      store8(resid + (size_t)row * D + c, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[i][e];
    }
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
  const float mean = sum / (float)D;
  float dsum = 0.f, dsq = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) {
      float d[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d[e] = v[i][e] - mean;
        dsum += d[e];
        dsq = fmaf(d[e], d[e], dsq);
      }
      store8(x16 + (size_t)row * D + c, d);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    dsum += __shfl_xor_sync(0xffffffff, dsum, o);
    dsq += __shfl_xor_sync(0xffffffff, dsq, o);
  }
  if (lane == 0) pivot[row] = mean;
  for (int j = lane; j < n_parts; j += 32)
    stats[(size_t)row * n_parts + j] = j == 0 ? make_float2(dsum, dsq) : make_float2(0.f, 0.f);
}

// One-time LayerNorm fold of a weight matrix W [rows, k] (fp16) consumed by
// LayerNorm(x) @ W^T + b:  W' = W * gamma (per column k, fp16), colsum[r] = sum_k W'[r, k]
// (of the fp16 values), b'[r] = b[r] + sum_k W[r, k] * beta[k].  One warp per output row.
// Output row r takes input row (r / hp) * hd + r % hp when r % hp < hd and is zero
// otherwise (heads of hd rows widened to hp; hd == hp is the identity).
__global__ void __launch_bounds__(256) fold_ln_kernel(const __half* __restrict__ w,
                                                      const float* __restrict__ b,
                                                      const float* __restrict__ gamma,
                                                      const float* __restrict__ beta, int rows_out,
                                                      int k, int hd, int hp,
                                                      __half* __restrict__ w_out,
                                                      float* __restrict__ b_out,
                                                      float* __restrict__ colsum) {
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (row >= rows_out) return;
  const int lane = lane_id();
  const int d = row % hp;
  if (d >= hd) {
    const float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int c = lane * 8; c < k; c += 256) store8(w_out + (size_t)row * k + c, z);
    if (lane == 0) {
      colsum[row] = 0.f;
      b_out[row] = 0.f;
    }
    return;
  }
  const int src = (row / hp) * hd + d;
  double cs = 0.0, bb = 0.0;
  for (int c = lane * 8; c < k; c += 256) {
    float wv[8], g[8], be[8], wf[8];
    load8<__half>(w + (size_t)src * k + c, wv);
    load8<float>(gamma + c, g);
    load8<float>(beta + c, be);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      wf[e] = __half2float(__float2half_rn(wv[e] * g[e]));
      cs += (double)wf[e];
      bb += (double)wv[e] * (double)be[e];
    }
    store8(w_out + (size_t)row * k + c, wf);
  }
  for (int o = 16; o > 0; o >>= 1) {
    cs += __shfl_xor_sync(0xffffffff, cs, o);
    bb += __shfl_xor_sync(0xffffffff, bb, o);
  }
  if (lane == 0) {
    colsum[row] = (float)cs;
    b_out[row] = (float)((double)b[src] + bb);
  }
}

// w [rows, cols] -> w_out [rows, (cols / hd) * hp]: column c of output row r is
// w[r, (c / hp) * hd + c % hp] when c % hp < hd, else 0.
__global__ void __launch_bounds__(256) pad_head_cols_kernel(const __half* __restrict__ w, int rows,
                                                            int cols, int hd, int hp,
                                                            __half* __restrict__ w_out) {
  const int cols_out = (cols / hd) * hp;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)rows * cols_out) return;
  const int r = (int)(i / cols_out), c = (int)(i - (long)r * cols_out);
  const int d = c % hp;
  w_out[i] = d < hd ? w[(size_t)r * cols + (c / hp) * hd + d] : __float2half_rn(0.f);
}

template <int VPL, typename TIn>
__global__ void __launch_bounds__(256) ln_rows_kernel(const TIn* __restrict__ in,
                                                      const int* __restrict__ rows_dev,
                                                      int rows_max, int D, const float* gamma,
                                                      const float* beta, float eps,
                                                      __half* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  const int row = blockIdx.x * (blockDim.x >> 5) + warp_id();
  const int rows = rows_dev ? min(*rows_dev, rows_max) : rows_max;
  if (row >= rows) return;
  const int lane = lane_id();
  float v[VPL][8];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) load8<TIn>(in + (size_t)row * D + c, v[i]);
  }
  ln_normalise<VPL>(v, D, gamma, beta, eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) store8(out + (size_t)row * D + c, v[i]);
  }
}

// Final LayerNorm over every output token; padded tokens are written as exact zeros.
// As the last kernel of a forward it also copies a non-zero device status word (a
// bounded wait of an earlier kernel of the forward gave up) into the caller's pinned
// host mirror, which the host reads without synchronising.
template <int VPL, typename TOut>
__global__ void __launch_bounds__(256) ln_final_scatter_kernel(const float* __restrict__ resid,
                                                               const int* __restrict__ dst_map,
                                                               int tokens, int D,
                                                               const float* gamma,
                                                               const float* beta, float eps,
                                                               TOut* __restrict__ out,
                                                               const int* status,
                                                               int* status_host) {
  griddep_wait();
  griddep_launch();
  if (blockIdx.x == 0 && threadIdx.x == 0 && status != nullptr && status_host != nullptr) {
    const int v = *reinterpret_cast<const volatile int*>(status);
    if (v != 0) *reinterpret_cast<volatile int*>(status_host) = v;
  }
  const int tok = blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (tok >= tokens) return;
  const int lane = lane_id();
  const int row = dst_map[tok];
  float v[VPL][8];
  if (row < 0) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = (lane + 32 * i) * 8;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
      if (c < D) store8(out + (size_t)tok * D + c, v[i]);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) load8<float>(resid + (size_t)row * D + c, v[i]);
  }
  ln_normalise<VPL>(v, D, gamma, beta, eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 8;
    if (c < D) store8(out + (size_t)tok * D + c, v[i]);
  }
}

// Self-test of the bounded wait: waits on an mbarrier that nothing arrives on, with
// a short limit, and reports TTTJ_DEV_TIMEOUT_SELFTEST.  Used by the failure
// detection test; it never hangs.
// With status_host (a plan's pinned mirror) the code is copied there too, as the last
// kernel of a forward would copy it.
__global__ void wait_timeout_selftest_kernel(int* status, int* status_host,
                                             unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!mbar_wait(smem_u32(&bar), 0, nullptr, limit_ns)) {
      report_status(status, TTTJ_DEV_TIMEOUT_SELFTEST);
      if (status_host != nullptr)
        *reinterpret_cast<volatile int*>(status_host) = TTTJ_DEV_TIMEOUT_SELFTEST;
    }
  }
}

}  // namespace tttj
