// Per-stage capture for numerics bisection (tttj_forward_debug): one sequence, one
// layer, the stages of the reference's capture_debug dump
// (kernels/sequence_resident.py:28-46, kernels/csrc/sequence_resident.cu:355-450):
// LN1 output, q, k, v, per-head scores and softmax probabilities, the attention output
// (P V), the output-projection branch and the FFN branch, each as fp32 [positions, ...]
// with zeros at padded positions.  The forward itself never materialises LN outputs,
// scores or probabilities (LayerNorm is folded into the GEMMs, attention keeps S and P
// in TMEM), so these small kernels recompute them from the captured rows; they are for
// debugging only and run on one sequence.
#include "launch.h"
#include "common.cuh"

namespace tttj {

namespace {

// dst[s][c] = src[row(s)][col_base + (c / hd) * hp + c % hd] for the sequence's valid
// positions s (row(s) = dst_map[b * S + s] >= 0), else 0.
__global__ void debug_gather_kernel(const void* src, int src_f16, int ld, int col_base, int cols,
                                    int hd, int hp, const int* dst_map, int b, int S, float* dst) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)S * cols) return;
  const int s = (int)(i / cols), c = (int)(i - (long)s * cols);
  const int row = dst_map[(size_t)b * S + s];
  float v = 0.f;
  if (row >= 0) {
    const size_t col = (size_t)col_base + (size_t)(c / hd) * hp + c % hd;
    v = src_f16 ? __half2float(static_cast<const __half*>(src)[(size_t)row * ld + col])
                : static_cast<const float*>(src)[(size_t)row * ld + col];
  }
  dst[i] = v;
}

// nn.LayerNorm of each valid row of x [S, D] (fp32, biased variance); padded rows 0.
__global__ void debug_ln_kernel(const float* x, const float* gamma, const float* beta, float eps,
                                int S, int D, const int* dst_map, int b, float* out) {
  const int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= S) return;
  const float* xr = x + (size_t)s * D;
  float* o = out + (size_t)s * D;
  if (dst_map[(size_t)b * S + s] < 0) {
    for (int c = lane; c < D; c += 32) o[c] = 0.f;
    return;
  }
  float sum = 0.f;
  for (int c = lane; c < D; c += 32) sum += xr[c];
  for (int k = 16; k > 0; k >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, k);
  const float mean = sum / (float)D;
  float sq = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float d = xr[c] - mean;
    sq += d * d;
  }
  for (int k = 16; k > 0; k >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, k);
  const float rstd = rsqrtf(sq / (float)D + eps);
  for (int c = lane; c < D; c += 32) o[c] = (xr[c] - mean) * rstd * gamma[c] + beta[c];
}

// scores[h][s][t] = q_h[s] . k_h[t] * scale, -inf where the key is padded or (causal)
// after the query; probs = softmax over t.  Rows of padded queries (and rows with no
// valid key) are written as zeros in both.
__global__ void debug_scores_kernel(const float* q, const float* k, const int* dst_map, int b,
                                    int S, int H, int hd, int causal, float scale, float* scores,
                                    float* probs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= H * S) return;
  const int h = i / S, s = i - h * S;
  const int D = H * hd;
  float* sr = scores + ((size_t)h * S + s) * S;
  float* pr = probs + ((size_t)h * S + s) * S;
  const bool qvalid = dst_map[(size_t)b * S + s] >= 0;
  float mx = -INFINITY;
  for (int t = 0; t < S; ++t) {
    const bool masked = !qvalid || dst_map[(size_t)b * S + t] < 0 || (causal && t > s);
    float v = -INFINITY;
    if (!masked) {
      float acc = 0.f;
      for (int d = 0; d < hd; ++d) acc = fmaf(q[(size_t)s * D + h * hd + d], k[(size_t)t * D + h * hd + d], acc);
      v = acc * scale;
      mx = fmaxf(mx, v);
    }
    sr[t] = qvalid ? v : 0.f;
  }
  float sum = 0.f;
  for (int t = 0; t < S; ++t) sum += (mx == -INFINITY || sr[t] == -INFINITY) ? 0.f : expf(sr[t] - mx);
  for (int t = 0; t < S; ++t)
    pr[t] = (sum > 0.f && sr[t] != -INFINITY && qvalid) ? expf(sr[t] - mx) / sum : 0.f;
}

__global__ void debug_diff_kernel(const float* a, const float* b, long n, float* out) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] - b[i];
}

inline int blocks(long n, int t) { return (int)((n + t - 1) / t); }

}  // namespace

cudaError_t debug_gather_launch(const void* src, int src_f16, int ld, int col_base, int cols, int hd,
                                int hp, const int* dst_map, int b, int S, float* dst,
                                cudaStream_t s) {
  debug_gather_kernel<<<blocks((long)S * cols, 256), 256, 0, s>>>(src, src_f16, ld, col_base, cols,
                                                                  hd, hp, dst_map, b, S, dst);
  return cudaGetLastError();
}

cudaError_t debug_ln_launch(const float* x, const float* gamma, const float* beta, float eps, int S,
                            int D, const int* dst_map, int b, float* out, cudaStream_t s) {
  debug_ln_kernel<<<blocks(S, 8), 256, 0, s>>>(x, gamma, beta, eps, S, D, dst_map, b, out);
  return cudaGetLastError();
}

cudaError_t debug_scores_launch(const float* q, const float* k, const int* dst_map, int b, int S,
                                int H, int hd, int causal, float scale, float* scores, float* probs,
                                cudaStream_t s) {
  debug_scores_kernel<<<blocks((long)H * S, 128), 128, 0, s>>>(q, k, dst_map, b, S, H, hd, causal,
                                                                scale, scores, probs);
  return cudaGetLastError();
}

cudaError_t debug_diff_launch(const float* a, const float* b, long n, float* out, cudaStream_t s) {
  debug_diff_kernel<<<blocks(n, 256), 256, 0, s>>>(a, b, n, out);
  return cudaGetLastError();
}

}  // namespace tttj
