// K2 (first generation): flash-style fused attention over the packed valid-token
// layout, warp-level mma.sync m16n8k16 (fp16 in, fp32 accumulate), online softmax in
// fp32 with exp2.
//
// Replaces BaselineSelfAttention's score/mask/softmax/PV sequence
// (benchmarks/torch_transformer_benchmark.py:97-117): scores = q k^T * hd^-0.5,
// causal mask triu(1) (:99-103), key-padding mask (:105-108), fp32 softmax (:111),
// probs @ v (:112).  Queries and keys are packed per sequence (only valid tokens), so
// the key-padding mask becomes "key index < valid length" and the causal mask
// compares packed positions, which preserve token order within a sequence.
//
// One CTA = 128 queries of one (sequence, head), 8 warps x 16 query rows; keys are
// streamed in 64-key tiles through a cp.async double buffer.  Key rows past the
// sequence's valid length are zero-filled in shared memory, so no other sequence's
// values (finite or not) can reach this sequence's output.
#pragma once
#include "common.cuh"
#include "params.h"

namespace tttj {

template <int HD>
struct AttnSmem {
  static constexpr int LD = HD + 8;  // padded row (halves) against ldmatrix bank conflicts
  static constexpr int Q_ELEMS = ATT_BM * LD;
  static constexpr int KV_ELEMS = ATT_BN * LD;
  static constexpr int BYTES = (Q_ELEMS + 4 * KV_ELEMS) * 2;
};

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;  // src-size 0 zero-fills the 16 destination bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Copy `nrows` rows of HD halves starting at packed row `row0` (column `col`) of
// the qkv buffer into shared memory; rows at or past `valid` are zero-filled.
template <int HD, int NROWS>
__device__ __forceinline__ void load_rows(uint32_t s_base, const __half* qkv, int ld, int row0,
                                          int col, int valid) {
  constexpr int CHUNKS = HD / 8;  // 16-byte chunks per row
  constexpr int TOTAL = NROWS * CHUNKS;
  for (int i = threadIdx.x; i < TOTAL; i += ATT_THREADS) {
    const int r = i / CHUNKS;
    const int c = i - r * CHUNKS;
    const bool ok = r < valid;
    const __half* src = qkv + (size_t)(row0 + (ok ? r : 0)) * ld + col + c * 8;
    cp_async_16(s_base + (uint32_t)((r * AttnSmem<HD>::LD + c * 8) * 2), src, ok);
  }
}

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(ATT_THREADS, 2) attention_mma_kernel(const AttnParams p) {
  using SM = AttnSmem<HD>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __half* sQ = reinterpret_cast<__half*>(smem_raw);
  __half* sK = sQ + SM::Q_ELEMS;      // 2 buffers
  __half* sV = sK + 2 * SM::KV_ELEMS;  // 2 buffers

  if ((int)blockIdx.x >= *p.item_count) return;
  const int2 item = p.items[blockIdx.x];
  const int b = item.x;
  const int q_tile = item.y >> 8;
  const int h = item.y & 0xff;
  const int seq0 = p.seq_off[b];
  const int len = p.seq_off[b + 1] - seq0;
  const int q0 = q_tile * ATT_BM;
  if (q0 >= len) return;
  const int q_valid = min(ATT_BM, len - q0);
  const int kv_end = CAUSAL ? min(len, q0 + ATT_BM) : len;
  const int n_kv = (kv_end + ATT_BN - 1) / ATT_BN;

  const int ld = 3 * p.d_model;
  const int qcol = h * HD;
  const int kcol = p.d_model + h * HD;
  const int vcol = 2 * p.d_model + h * HD;

  const uint32_t sQa = smem_u32(sQ);
  const uint32_t sKa = smem_u32(sK);
  const uint32_t sVa = smem_u32(sV);
  constexpr uint32_t KV_BYTES = SM::KV_ELEMS * 2;

  load_rows<HD, ATT_BM>(sQa, p.qkv, ld, seq0 + q0, qcol, q_valid);
  load_rows<HD, ATT_BN>(sKa, p.qkv, ld, seq0, kcol, kv_end);
  load_rows<HD, ATT_BN>(sVa, p.qkv, ld, seq0, vcol, kv_end);
  cp_async_commit();

  const int warp = warp_id();
  const int lane = lane_id();
  const int g = lane >> 2;  // row within the 8-row group
  const int t = lane & 3;   // column pair

  // Query rows owned by this thread (relative to the sequence).
  const int qr0 = q0 + warp * 16 + g;
  const int qr1 = qr0 + 8;

  uint32_t qf[HD / 16][4];
  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int it = 0; it < n_kv; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_kv) {
      const int k0n = (it + 1) * ATT_BN;
      load_rows<HD, ATT_BN>(sKa + (buf ^ 1) * KV_BYTES, p.qkv, ld, seq0 + k0n, kcol, kv_end - k0n);
      load_rows<HD, ATT_BN>(sVa + (buf ^ 1) * KV_BYTES, p.qkv, ld, seq0 + k0n, vcol, kv_end - k0n);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    if (it == 0) {
#pragma unroll
      for (int kc = 0; kc < HD / 16; ++kc) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kc * 16 + (lane >> 4) * 8;
        ldsm_x4(sQa + (uint32_t)((r * SM::LD + c) * 2), qf[kc][0], qf[kc][1], qf[kc][2],
                qf[kc][3]);
      }
    }

    // S = Q K^T for this warp's 16 rows x 64 keys.
    float s[ATT_BN / 8][4];
#pragma unroll
    for (int j = 0; j < ATT_BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t kbase = sKa + buf * KV_BYTES;
#pragma unroll
    for (int kc = 0; kc < HD / 16; ++kc) {
#pragma unroll
      for (int jp = 0; jp < ATT_BN / 16; ++jp) {
        const int key = jp * 16 + (lane & 7) + (lane >> 4) * 8;
        const int dim = kc * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + (uint32_t)((key * SM::LD + dim) * 2), b0, b1, b2, b3);
        mma_16816(s[2 * jp], qf[kc], b0, b1);
        mma_16816(s[2 * jp + 1], qf[kc], b2, b3);
      }
    }

    // Masking: key index (relative to the sequence) must be < kv_end and, if causal,
    // <= the query index.  Only the last tile and diagonal tiles need it.
    const int k0 = it * ATT_BN;
    const bool need_mask = (k0 + ATT_BN > kv_end) || (CAUSAL && k0 + ATT_BN - 1 > q0 + warp * 16);
    if (need_mask) {
#pragma unroll
      for (int j = 0; j < ATT_BN / 8; ++j) {
        const int kc0 = k0 + j * 8 + 2 * t;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kk = kc0 + e;
          const bool bad0 = kk >= kv_end || (CAUSAL && kk > qr0);
          const bool bad1 = kk >= kv_end || (CAUSAL && kk > qr1);
          if (bad0) s[j][e] = -INFINITY;
          if (bad1) s[j][2 + e] = -INFINITY;
        }
      }
    }

    // Online softmax (base 2).
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < ATT_BN / 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
    const float mn0 = fmaxf(m0, mx0 * p.scale_log2);
    const float mn1 = fmaxf(m1, mx1 * p.scale_log2);
    // A row that has seen only masked keys keeps a finite base so exp2 never sees inf-inf.
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float alpha0 = exp2f(m0 - base0);
    const float alpha1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;

    uint32_t pf[ATT_BN / 16][4];
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < ATT_BN / 8; ++j) {
      const float p0 = exp2f(s[j][0] * p.scale_log2 - base0);
      const float p1 = exp2f(s[j][1] * p.scale_log2 - base0);
      const float p2 = exp2f(s[j][2] * p.scale_log2 - base1);
      const float p3 = exp2f(s[j][3] * p.scale_log2 - base1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      // C fragment of key block j becomes half of the A fragment of k-chunk j/2.
      pf[j >> 1][(j & 1) * 2 + 0] = pack_half2(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_half2(p2, p3);
    }
    l0 = l0 * alpha0 + rs0;
    l1 = l1 * alpha1 + rs1;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= alpha0;
      o[i][1] *= alpha0;
      o[i][2] *= alpha1;
      o[i][3] *= alpha1;
    }

    // O += P V.
    const uint32_t vbase = sVa + buf * KV_BYTES;
#pragma unroll
    for (int kc = 0; kc < ATT_BN / 16; ++kc) {
#pragma unroll
      for (int np = 0; np < HD / 16; ++np) {
        const int key = kc * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int dim = np * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + (uint32_t)((key * SM::LD + dim) * 2), b0, b1, b2, b3);
        mma_16816(o[2 * np], pf[kc], b0, b1);
        mma_16816(o[2 * np + 1], pf[kc], b2, b3);
      }
    }
    __syncthreads();
  }

  // Row sums across the quad, normalise, store valid rows.
  l0 += __shfl_xor_sync(0xffffffff, l0, 1);
  l0 += __shfl_xor_sync(0xffffffff, l0, 2);
  l1 += __shfl_xor_sync(0xffffffff, l1, 1);
  l1 += __shfl_xor_sync(0xffffffff, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  __half* out0 = p.ctx + (size_t)(seq0 + qr0) * p.d_model + h * HD;
  __half* out1 = p.ctx + (size_t)(seq0 + qr1) * p.d_model + h * HD;
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) {
    const int col = i * 8 + 2 * t;
    if (qr0 < len)
      *reinterpret_cast<uint32_t*>(out0 + col) = pack_half2(o[i][0] * inv0, o[i][1] * inv0);
    if (qr1 < len)
      *reinterpret_cast<uint32_t*>(out1 + col) = pack_half2(o[i][2] * inv1, o[i][3] * inv1);
  }
}

}  // namespace tttj
