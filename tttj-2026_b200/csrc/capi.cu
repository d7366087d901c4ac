// C ABI of the forward path (include/tttj_b200.h): configuration checks, packed
// weight and workspace layouts, TMA descriptor construction, the plan object and the
// per-layer launch sequence.
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tttj_b200.h"
#include "launch.h"

using namespace tttj;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TTTJ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define TTTJ_CUDA(call)                                   \
  do {                                                    \
    cudaError_t e_ = (call);                              \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);   \
  } while (0)

constexpr size_t kAlign = 256;
inline size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }
constexpr float kLnEps = 1e-5f;  // nn.LayerNorm default (torch_transformer_benchmark.py:128)
constexpr unsigned long long kWaitLimitNs = TTTJ_WAIT_LIMIT_NS;

// ---------------------------------------------------------------- head layout
// The attention kernels handle head_dim 32, 64, 128 and 256.  Narrower heads (and
// widths between those) are padded: the plan's folded QKV weights put head h's
// q / k / v columns at h * hp .. h * hp + hd - 1 of a layout head of hp columns, whose
// other columns are zero rows of the weight (so q, k, v and the attention output are
// zero there), and the out_proj weight gets matching zero columns.  Scores and
// outputs are unchanged; the softmax scale stays hd^-0.5.
int layout_hd(int hd) { return hd <= 32 ? 32 : hd <= 64 ? 64 : hd <= 128 ? 128 : 256; }
int head_dim_of(const tttj_config& c) { return c.d_model / c.num_heads; }
int layout_hd(const tttj_config& c) { return layout_hd(head_dim_of(c)); }
// Columns of each of the q | k | v blocks in the workspace (= d_model unless padded).
size_t qkv_width(const tttj_config& c) { return (size_t)c.num_heads * layout_hd(c); }
bool heads_padded(const tttj_config& c) { return layout_hd(c) != head_dim_of(c); }

// ---------------------------------------------------------------- weights layout
size_t field_bytes(const tttj_config& c, int field) {
  const size_t D = c.d_model, F = c.ffn_dim;
  switch (field) {
    case TTTJ_W_QKV: return 3 * D * D * 2;
    case TTTJ_W_OUT: return D * D * 2;
    case TTTJ_W_FFN_IN: return F * D * 2;
    case TTTJ_W_FFN_OUT: return D * F * 2;
    case TTTJ_B_QKV: return 3 * D * 4;
    case TTTJ_B_OUT: return D * 4;
    case TTTJ_B_FFN_IN: return F * 4;
    case TTTJ_B_FFN_OUT: return D * 4;
    case TTTJ_LN1_W: case TTTJ_LN1_B: case TTTJ_LN2_W: case TTTJ_LN2_B:
    case TTTJ_LNF_W: case TTTJ_LNF_B: return D * 4;
    default: return 0;
  }
}

size_t layer_stride(const tttj_config& c) {
  size_t s = 0;
  for (int f = TTTJ_W_QKV; f <= TTTJ_LN2_B; ++f) s += align_up(field_bytes(c, f));
  return s;
}

bool weight_offset(const tttj_config& c, int layer, int field, size_t* off, size_t* bytes) {
  if (layer < 0 || layer > c.num_layers) return false;
  if (layer == c.num_layers) {
    if (field != TTTJ_LNF_W && field != TTTJ_LNF_B) return false;
    *off = (size_t)c.num_layers * layer_stride(c) +
           (field == TTTJ_LNF_B ? align_up(field_bytes(c, TTTJ_LNF_W)) : 0);
    *bytes = field_bytes(c, field);
    return true;
  }
  if (field < TTTJ_W_QKV || field > TTTJ_LN2_B) return false;
  size_t o = (size_t)layer * layer_stride(c);
  for (int f = TTTJ_W_QKV; f < field; ++f) o += align_up(field_bytes(c, f));
  *off = o;
  *bytes = field_bytes(c, field);
  return true;
}

// ---------------------------------------------------------------- workspace layout
struct WsLayout {
  size_t seq_len, seq_off, packed_src, dst_map, items, item_count, counters, status;
  size_t attn_plan;  // split plans: token plan of the whole sequence's attention
  size_t resid, x16, qkv, ctx, hid, stats, pivot;
  size_t total;
};

// Per-layer fold region: Wqkv' [3Q, D] fp16 (Q = qkv_width), W1' [F, D] fp16, then
// fp32 vectors bqkv' [3Q], colsum_qkv [3Q], b1' [F], colsum_1 [F], and for padded heads
// the out_proj weight with zero columns Wo' [D, Q] fp16.
struct FoldLayout {
  size_t wqkv, w1, bqkv, cqkv, b1, c1, wo, total;
};
// Statistics partials per row produced by a residual GEMM (N = d_model): two column
// halves per column tile (a half past d_model writes zeros).  Tiles are at least 64
// columns wide, so 2 * ceil(d_model / 64) bounds the count.
int stats_parts(const tttj_config& c) { return 2 * ((c.d_model + 63) / 64); }  // upper bound

FoldLayout fold_layout(const tttj_config& c) {
  const size_t D = c.d_model, F = c.ffn_dim, Q = qkv_width(c);
  FoldLayout f{};
  size_t o = 0;
  f.wqkv = o; o += align_up(3 * Q * D * 2);
  f.w1 = o; o += align_up(F * D * 2);
  f.bqkv = o; o += align_up(3 * Q * 4);
  f.cqkv = o; o += align_up(3 * Q * 4);
  f.b1 = o; o += align_up(F * 4);
  f.c1 = o; o += align_up(F * 4);
  f.wo = o; o += heads_padded(c) ? align_up(D * Q * 2) : 0;
  f.total = o;
  return f;
}

// Work items of 128 query rows bound every item size.
size_t attn_items_max(size_t B, size_t S, size_t H) {
  return B * H * ((S + ATC_BM - 1) / ATC_BM);
}

// Token-plan part of the workspace (shared by the forward and tttj_attention).
size_t plan_layout(size_t B, size_t S, size_t H, WsLayout* w) {
  const size_t T = B * S;
  size_t o = 0;
  w->seq_len = o; o += align_up(B * 4);
  w->seq_off = o; o += align_up((B + 1) * 4);
  w->packed_src = o; o += align_up(T * 4);
  w->dst_map = o; o += align_up(T * 4);
  w->items = o; o += align_up(attn_items_max(B, S, H) * 8);
  w->item_count = o; o += align_up(4);
  w->counters = o; o += align_up(4 * PLAN_COUNTERS);
  w->status = o; o += align_up(4);
  return o;
}

// full_rows > 0: a split plan (one sequence whose tokens are shared out between ranks):
// the rank's own rows (T = seq_len of the config) everywhere, except qkv and ctx, which
// hold the whole sequence (full_rows rows, the rank's at their sequence positions), and
// a second token plan for the whole sequence's attention.
WsLayout ws_layout(const tttj_config& c, size_t full_rows = 0) {
  WsLayout w{};
  const size_t T = (size_t)c.batch_size * c.seq_len, D = c.d_model, F = c.ffn_dim;
  const size_t Q = qkv_width(c);
  size_t o = plan_layout(c.batch_size, c.seq_len, c.num_heads, &w);
  if (full_rows) {
    WsLayout wa{};
    w.attn_plan = o;
    o += plan_layout(1, full_rows, c.num_heads, &wa);
  }
  const size_t TQ = full_rows ? full_rows : T;
  w.resid = o; o += align_up(T * D * 4);
  w.x16 = o; o += align_up(T * D * 2);
  w.qkv = o; o += align_up(TQ * 3 * Q * 2);
  w.ctx = o; o += align_up(TQ * Q * 2);
  w.hid = o; o += align_up(T * F * 2);
  w.stats = o; o += align_up((size_t)2 * T * stats_parts(c) * 8);
  w.pivot = o; o += align_up((size_t)2 * T * 4);
  w.total = o;
  return w;
}

// The LayerNorm-folded weights (FoldLayout per layer) depend on the configuration's
// layer shapes only, not on batch or sequence length: one buffer per module, shared
// by every plan.
size_t folded_bytes(const tttj_config& c) { return (size_t)c.num_layers * fold_layout(c).total; }

TokenPlan token_plan_at(uint8_t* base, const WsLayout& w) {
  TokenPlan tp;
  tp.seq_len = reinterpret_cast<int*>(base + w.seq_len);
  tp.seq_off = reinterpret_cast<int*>(base + w.seq_off);
  tp.packed_src = reinterpret_cast<int*>(base + w.packed_src);
  tp.dst_map = reinterpret_cast<int*>(base + w.dst_map);
  tp.items = reinterpret_cast<int2*>(base + w.items);
  tp.item_count = reinterpret_cast<int*>(base + w.item_count);
  tp.counters = reinterpret_cast<int*>(base + w.counters);
  return tp;
}

// ---------------------------------------------------------------- TMA descriptors
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major matrix [rows, cols] with row stride `ld` elements, moved in boxes of
// box_cols x box_rows elements.
int make_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dtype, uint32_t elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(TTTJ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * elem_bytes) % 16)
    return fail(TTTJ_ERR_INVALID, "TMA operand must be 16-byte aligned with a 16-byte row stride");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TTTJ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TTTJ_OK;
}

// Per-layer 2-D matrices [rows, cols] (row stride `ld` elements) laid out `layer_bytes`
// apart, as one 3-D tensor {cols, rows, layers} moved in boxes of box_cols x box_rows.
int make_tmap_3d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                 uint64_t layers, uint64_t layer_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(TTTJ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16 || layer_bytes % 16)
    return fail(TTTJ_ERR_INVALID, "TMA operand must be 16-byte aligned with 16-byte strides");
  cuuint64_t dims[3] = {cols, rows, layers};
  cuuint64_t strides[2] = {ld * 2, layer_bytes};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TTTJ_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return TTTJ_OK;
}

// GEMM operand: fp16 [rows, cols], boxes of 64 columns (128 B, one swizzle atom) x
// box_rows rows, 128-byte swizzle (the canonical K-major UMMA layout).
int make_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
              uint32_t box_rows) {
  return make_tmap_2d(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, rows, cols, ld, 64, box_rows,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

// TMA map + parameters of the tcgen05 attention over a packed qkv buffer of
// `qkv_rows` rows with H heads of `hp` layout columns (hd of them real): boxes of
// min(hp, 64) columns x 128 rows, swizzle = the box row width.
int build_attention(CUtensorMap* tm, AtcParams* ap, int* grid, const void* qkv, void* ctx,
                    int qkv_rows, int B, int S, int H, int hd, int hp, const TokenPlan& tp,
                    int* status, int num_sms) {
  const int width = H * hp;
  const uint32_t box_cols = hp < 64 ? (uint32_t)hp : 64u;
  int rc = make_tmap_2d(tm, qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)qkv_rows,
                        (uint64_t)(3 * width), (uint64_t)(3 * width), box_cols, ATC_BM,
                        box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  ap->seq_off = tp.seq_off;
  ap->items = tp.items;
  ap->item_count = tp.item_count;
  ap->work_counter = tp.counters;  // the forward points layer l at counters[l]
  ap->ctx = static_cast<__half*>(ctx);
  ap->rows_max = qkv_rows;
  ap->qkv_width = width;
  ap->scale_log2 = (1.0f / sqrtf((float)hd)) * 1.4426950408889634f;
  ap->status = status;
  ap->wait_limit_ns = kWaitLimitNs;
  const int item_rows = atc_item_rows(hp);
  const long items = (long)B * H * ((S + item_rows - 1) / item_rows);
  *grid = (int)(items < num_sms ? items : num_sms);
  return TTTJ_OK;
}

int sm_count(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  return n;
}

int build_gemm(GemmLaunch* g, const void* a, int lda, const void* w, int ldw, const float* bias,
               void* out, int ldo, const void* residual, int ldr, int rows, const int* rows_dev,
               int n, int k, int epi, int* status, int num_sms) {
  if (n <= 0 || k <= 0 || rows < 0) return fail(TTTJ_ERR_INVALID, "linear: bad sizes");
  if (n % 32 != 0) return fail(TTTJ_ERR_INVALID, "linear: n=%d must be a multiple of 32", n);
  // k need not fill the last 64-column block: TMA zero-fills columns past k.
  if (k % 8 != 0) return fail(TTTJ_ERR_INVALID, "linear: k=%d must be a multiple of 8", k);
  const bool has_res = epi == EPI_BIAS_RESIDUAL || epi == EPI_BIAS_RESIDUAL_F32 ||
                       epi == EPI_RESIDUAL_F32_STATS;
  if (lda % 8 || ldw % 8 || ldo % 8 || (has_res && ldr % 8))
    return fail(TTTJ_ERR_INVALID, "linear: row strides must be multiples of 8 elements");
  if (epi < EPI_BIAS || epi > EPI_LN_FOLD_GELU)
    return fail(TTTJ_ERR_INVALID, "linear: unknown epilogue %d", epi);
  if (has_res && residual == nullptr)
    return fail(TTTJ_ERR_INVALID, "linear: residual epilogue needs a residual");
  if ((reinterpret_cast<uintptr_t>(bias) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(residual) & 15))
    return fail(TTTJ_ERR_INVALID, "linear: bias/out/residual must be 16-byte aligned");
  if (num_sms <= 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    num_sms = sm_count(dev);
    if (num_sms <= 0) return fail(TTTJ_ERR_CUDA, "could not query the SM count");
  }
  std::memset(g, 0, sizeof(*g));
  gemm_choose(rows, n, k, epi, num_sms, &g->bn, &g->pair);
  g->rbuf = gemm_choose_rbuf(g->bn, g->pair, k, epi, residual == out && ldr == ldo);
  g->epiw = gemm_choose_epiw(g->bn, epi, g->rbuf);
  g->epi = epi;
  int rc = make_tmap(&g->tmA, a, (uint64_t)(rows > 0 ? rows : 1), (uint64_t)k, (uint64_t)lda, GEMM_BM);
  if (rc) return rc;
  // B boxes: bn rows, or bn / 2 per CTA of a pair.
  rc = make_tmap(&g->tmB, w, (uint64_t)n, (uint64_t)k, (uint64_t)ldw,
                 (uint32_t)(g->pair ? g->bn / 2 : g->bn));
  if (rc) return rc;
  // Output: 32x32 boxes; fp32 rows of the box are 128 B (128-byte swizzle), fp16 rows
  // 64 B (64-byte swizzle), matching the epilogue's staging layout.
  if (epi == EPI_BIAS_RESIDUAL_F32 || epi == EPI_RESIDUAL_F32_STATS)
    rc = make_tmap_2d(&g->tmC, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, (uint64_t)(rows > 0 ? rows : 1),
                      (uint64_t)n, (uint64_t)ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  else
    rc = make_tmap_2d(&g->tmC, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)(rows > 0 ? rows : 1),
                      (uint64_t)n, (uint64_t)ldo, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  g->p.rows_dev = rows_dev;
  g->p.rows_max = rows;
  g->p.n = n;
  g->p.k = k;
  g->p.bias = bias;
  g->p.out = out;
  g->p.ldo = ldo;
  g->p.residual = residual;
  g->p.ldr = ldr;
  g->p.status = status;
  g->p.wait_limit_ns = kWaitLimitNs;
  const long tm = g->pair ? 2 * GEMM_BM : GEMM_BM;
  const long tiles = (long)((rows + tm - 1) / tm) * ((n + g->bn - 1) / g->bn);
  if (g->pair) {
    const long pairs = num_sms / 2;
    g->grid = 2 * (int)(tiles < pairs ? tiles : pairs);
  } else {
    g->grid = (int)(tiles < num_sms ? tiles : num_sms);
  }
  return TTTJ_OK;
}

int check_config(const tttj_config* c) {
  if (!c) return fail(TTTJ_ERR_INVALID, "null config");
  if (c->batch_size <= 0 || c->seq_len <= 0 || c->d_model <= 0 || c->num_heads <= 0 ||
      c->ffn_dim <= 0 || c->num_layers <= 0)
    return fail(TTTJ_ERR_INVALID, "config fields must be positive");
  if (c->d_model % c->num_heads != 0)
    return fail(TTTJ_ERR_INVALID, "d_model (%d) must be divisible by num_heads (%d)", c->d_model,
                c->num_heads);
  const int hd = c->d_model / c->num_heads;
  if (hd % 8 != 0 || hd > 256)
    return fail(TTTJ_ERR_INVALID,
                "no B200 kernel for head_dim=%d (supported: multiples of 8 up to 256)", hd);
  if (c->d_model % 32 != 0 || c->ffn_dim % 32 != 0)
    return fail(TTTJ_ERR_INVALID, "d_model (%d) and ffn_dim (%d) must be multiples of 32",
                c->d_model, c->ffn_dim);
  if (c->d_model > 2048) return fail(TTTJ_ERR_INVALID, "d_model=%d exceeds 2048", c->d_model);
  if (c->num_heads > 255) return fail(TTTJ_ERR_INVALID, "num_heads=%d exceeds 255", c->num_heads);
  if (c->num_layers > PLAN_COUNTERS)
    return fail(TTTJ_ERR_INVALID, "num_layers=%d exceeds %d", c->num_layers, PLAN_COUNTERS);
  const long long T = (long long)c->batch_size * c->seq_len;
  const long long widest = c->ffn_dim > 3ll * c->num_heads * layout_hd(hd)
                               ? c->ffn_dim : 3ll * c->num_heads * layout_hd(hd);
  if (T * widest >= (1ll << 40) ||
      T >= (1ll << 31) - 256)
    return fail(TTTJ_ERR_INVALID, "batch_size*seq_len too large");
  // Token plan shared memory (rows.cuh plan_tokens_kernel): ints plus mask staging.
  const long long plan_smem =
      4ll * (2ll * c->batch_size + 3 + (c->seq_len + ATC_BN - 1) / ATC_BN + 1 + 3) +
      512ll * (PLAN_THREADS / 32);
  if (plan_smem > 200 * 1024) return fail(TTTJ_ERR_INVALID, "batch_size/seq_len too large for the token plan");
  return TTTJ_OK;
}

// Shapes the resident-stack kernel (resident.cuh) takes: sequences of <= 128 tokens,
// the residual (d_model fp32 columns) plus the largest step accumulator inside TMEM's
// 512 columns, residual MMA groups of d_model <= 128 or two of 128, and the shared
// memory layout within the 227 KB per CTA.
// TMEM columns a resident step needs after the residual, for `gh` heads per step.
int resident_acc_cols(int hp, int gh, int F) {
  const int fc = F < 128 ? F : 128;
  int acc = 3 * gh * hp;                                  // q | k | v
  if (gh * (128 + hp) > acc) acc = gh * (128 + hp);       // S (P over it) and O
  return fc > acc ? fc : acc;                             // one FFN chunk
}
// Heads per attention step: pairs for hp 32 with an even head count when TMEM allows.
int resident_gh(const tttj_config& c) {
  const int hp = layout_hd(c);
  return (hp == 32 && c.num_heads % 2 == 0 &&
          c.d_model + resident_acc_cols(hp, 2, c.ffn_dim) <= 512) ? 2 : 1;
}
bool resident_fits(const tttj_config& c) {
  const int D = c.d_model, hp = layout_hd(c), F = c.ffn_dim;
  if (c.seq_len > RES_ROWS) return false;
  if (!(D <= 128 || D == 256) || D % 32) return false;
  if (hp != 32 && hp != 64 && hp != 128) return false;
  const int gh = resident_gh(c);
  if (D + resident_acc_cols(hp, gh, F) > 512) return false;
  return res_layout(D, F, hp, c.num_heads * hp, gh).stages >= 3;
}

// Whether TTTJ_PATH_AUTO takes the resident kernel for a shape it fits.  One CTA works
// through 3H / gh + 3 + ceil(F / 128) worker <-> MMA hand-offs per layer (about 1.5 us
// each) and streams every layer's weights through its own ring (about 60 GB/s);
// measured on B200 against the layer-by-layer kernels, the resident kernel is faster up
// to about 32 hand-offs and 768 KB of weights per layer (the reference's cases 1-7 and
// 9-12; case 11 with 16 heads: 0.202 vs 0.224 ms) and slower beyond (C1, 1.6 MB of
// weights per layer: 0.156 vs 0.076 ms).
bool resident_preferred(const tttj_config& c) {
  const long D = c.d_model, F = c.ffn_dim, Q = (long)qkv_width(c);
  const long steps = 3l * c.num_heads / resident_gh(c) + 3 + (F + 127) / 128;
  const long weight_bytes = 2 * (3 * Q * D + D * Q + 2 * D * F);
  return steps <= 32 && weight_bytes <= 768 * 1024;
}

struct LayerGemms {
  GemmLaunch qkv, out, ffn_in, ffn_out;
  const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
};

}  // namespace

struct tttj_plan {
  tttj_config cfg;
  int device;
  int num_sms;
  const uint8_t* weights;
  const uint8_t* folded;  // LayerNorm-folded weights (tttj_fold_weights), per layer
  size_t fold_layer;      // bytes per layer of `folded`
  uint8_t* ws;
  WsLayout lay;
  TokenPlan tp;
  int* status;
  // Pinned, device-mapped mirror of the status word: the last kernel of every forward
  // copies a non-zero device status into it, and the next forward reads it without
  // synchronising.
  int* status_host = nullptr;
  // Cross-stream ordering of the plan's workspace: completion of the last forward and
  // the stream it ran on.  A forward on another stream first waits for it.
  cudaEvent_t done = nullptr;
  cudaStream_t last_stream = nullptr;
  bool has_last = false;
  float* resid;  // fp32 residual stream
  __half *x16, *qkv, *ctx, *hid;  // x16: fp16 copy of resid - pivot (GEMM A operand)
  float2* stats;  // [2][T][parts] LayerNorm statistics partials: LN1 (next QKV), LN2 (ffn_in)
  float* pivot;   // [2][T] per-row pivot of each statistics buffer
  // Split plan (tttj_plan_create_cp): this rank runs rows [cp_lo, cp_lo + T) of one
  // sequence of cp_len valid tokens; qkv / ctx hold cp_full rows of the whole sequence.
  bool cp = false;
  int cp_lo = 0, cp_len = 0, cp_full = 0;
  TokenPlan tp_attn;  // the whole sequence's attention items (this rank's queries)
  int parts;      // statistics partials per row of LN1 (ffn_out, the gather -> QKV)
  int parts_ln2;  // ... of LN2 (out_proj -> ffn_in)
  std::vector<LayerGemms> layers;
  const float *lnf_w, *lnf_b;
  CUtensorMap attn_tm;
  AtcParams attn;
  int attn_grid;
  // Resident-stack path (sequences of <= 128 tokens), built when the shape fits.
  // The token plan in the workspace is the all-valid one (the last forward had no mask):
  // a forward without a mask skips the plan kernel.  The gather kernel, first of every
  // layer-by-layer forward, zeroes the attention work counters.
  bool plan_static = false;
  bool captured = false;     // a forward of this plan was captured into a CUDA graph
  bool res_ok = false;       // the resident kernel fits this shape (launch built)
  bool res_auto = false;     // ... and TTTJ_PATH_AUTO prefers it
  int path = TTTJ_PATH_AUTO;
  ResLaunch res;
  // Optional per-kernel-class timing (tttj_plan_enable_timing).
  bool timing = false;
  std::vector<cudaEvent_t> ev_start, ev_stop;  // one pair per launch of one forward
  std::vector<int> ev_class;
  size_t ev_used = 0;
  double class_ms[TTTJ_KCLASS_COUNT] = {};
  long class_launches[TTTJ_KCLASS_COUNT] = {};
};

namespace {
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};
}  // namespace

int layerwise_launches(const tttj_config& c) { return 5 * c.num_layers + 3; }
// Most launches one forward of a plan may record (a split plan's first has two plans).
int max_launches(const tttj_config& c) { return layerwise_launches(c) + 1; }
bool use_resident(const tttj_plan* p) {
  return p->path == TTTJ_PATH_RESIDENT || (p->path == TTTJ_PATH_AUTO && p->res_auto);
}
int launches_per_forward(const tttj_plan* p) {
  if (p->cp) return layerwise_launches(p->cfg) - 1 + (p->plan_static ? 0 : 2);
  return use_resident(p) ? 1 : layerwise_launches(p->cfg) - (p->plan_static ? 1 : 0);
}

// Fold the events of the previous timed forward into the per-class totals.
int collect_timing(tttj_plan* p) {
  if (p->ev_used == 0) return TTTJ_OK;
  TTTJ_CUDA(cudaEventSynchronize(p->ev_stop[p->ev_used - 1]));
  for (size_t i = 0; i < p->ev_used; ++i) {
    float ms = 0.f;
    TTTJ_CUDA(cudaEventElapsedTime(&ms, p->ev_start[i], p->ev_stop[i]));
    p->class_ms[p->ev_class[i]] += ms;
    p->class_launches[p->ev_class[i]] += 1;
  }
  p->ev_used = 0;
  return TTTJ_OK;
}

void destroy_events(tttj_plan* p) {
  for (auto e : p->ev_start) cudaEventDestroy(e);
  for (auto e : p->ev_stop) cudaEventDestroy(e);
  p->ev_start.clear();
  p->ev_stop.clear();
  p->ev_class.clear();
  p->ev_used = 0;
}

// Host-side resources of a plan (the device memory is the caller's).  Waits for the
// plan's last forward first, so that the caller may free or reuse the workspace once
// the plan is destroyed.
void plan_release(tttj_plan* p) {
  if (p->done) {
    if (p->has_last) cudaEventSynchronize(p->done);
    cudaEventDestroy(p->done);
    p->done = nullptr;
  }
  destroy_events(p);
  if (p->status_host) {
    cudaFreeHost(p->status_host);
    p->status_host = nullptr;
  }
}

// TMA maps and parameters of the resident-stack kernel: the plan's folded QKV / ffn_in
// weights and (for padded heads) padded out_proj weight in the workspace, the caller's
// out_proj / ffn_out weights, all as 3-D maps over the layers.
int build_resident(tttj_plan* p, const FoldLayout& fl) {
  const tttj_config& c = p->cfg;
  const int D = c.d_model, F = c.ffn_dim, hp = layout_hd(c), Q = (int)qkv_width(c), L = c.num_layers;
  const int gh = resident_gh(c);
  const ResLayout ly = res_layout(D, F, hp, Q, gh);
  const uint8_t* fold = p->folded;
  const size_t fstride = p->fold_layer, lstride = layer_stride(c);
  auto W = [&](int field) -> const uint8_t* {
    size_t off = 0, bytes = 0;
    weight_offset(c, 0, field, &off, &bytes);
    return p->weights + off;
  };
  ResLaunch& r = p->res;
  std::memset(&r, 0, sizeof(r));
  // Wqkv boxes: the q (k, v) rows of the gh heads of one attention step.
  int rc = make_tmap_3d(&r.tmWqkv, fold + fl.wqkv, (uint64_t)3 * Q, D, D, L, fstride, 64,
                        (uint32_t)(ly.qkv_merged ? gh * hp : hp), CU_TENSOR_MAP_SWIZZLE_128B);
  const uint32_t woc = hp < 64 ? hp : 64;
  const CUtensorMapSwizzle wosw = hp < 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  if (!rc) {
    if (heads_padded(c))
      rc = make_tmap_3d(&r.tmWo, fold + fl.wo, D, Q, Q, L, fstride, woc, ly.NB, wosw);
    else
      rc = make_tmap_3d(&r.tmWo, W(TTTJ_W_OUT), D, D, D, L, lstride, woc, ly.NB, wosw);
  }
  if (!rc)
    rc = make_tmap_3d(&r.tmW1, fold + fl.w1, F, D, D, L, fstride, 64, ly.FC, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc)
    rc = make_tmap_3d(&r.tmW2, W(TTTJ_W_FFN_OUT), D, F, F, L, lstride, 64, ly.NB,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  ResParams& q = r.p;
  q.B = c.batch_size;
  q.S = c.seq_len;
  q.D = D;
  q.H = c.num_heads;
  q.F = F;
  q.L = L;
  q.causal = c.causal ? 1 : 0;
  q.hp = hp;
  q.gh = gh;
  q.Q = Q;
  q.scale_log2 = (1.0f / sqrtf((float)head_dim_of(c))) * 1.4426950408889634f;
  q.eps = kLnEps;
  q.bqkv = reinterpret_cast<const float*>(fold + fl.bqkv);
  q.cqkv = reinterpret_cast<const float*>(fold + fl.cqkv);
  q.b1 = reinterpret_cast<const float*>(fold + fl.b1);
  q.c1 = reinterpret_cast<const float*>(fold + fl.c1);
  q.fold_stride = fstride;
  q.bo = reinterpret_cast<const float*>(W(TTTJ_B_OUT));
  q.b2 = reinterpret_cast<const float*>(W(TTTJ_B_FFN_OUT));
  q.layer_stride = lstride;
  q.lnf_w = p->lnf_w;
  q.lnf_b = p->lnf_b;
  q.status = p->status;
  q.status_host = p->status_host;
  q.wait_limit_ns = kWaitLimitNs;
  p->res_ok = true;
  p->res_auto = resident_preferred(c);
  return TTTJ_OK;
}

extern "C" {

const char* tttj_last_error(void) { return g_last_error.c_str(); }

const char* tttj_version(void) { return "tttj_b200 0.1 (sm_100a)"; }

int tttj_validate_config(const tttj_config* cfg) { return check_config(cfg); }

size_t tttj_weights_bytes(const tttj_config* cfg) {
  if (check_config(cfg)) return 0;
  size_t off, bytes;
  weight_offset(*cfg, cfg->num_layers, TTTJ_LNF_B, &off, &bytes);
  return align_up(off + bytes);
}

int tttj_weight_offset(const tttj_config* cfg, int layer, int field, size_t* offset,
                       size_t* bytes) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (!offset || !bytes) return fail(TTTJ_ERR_INVALID, "null output pointer");
  if (!weight_offset(*cfg, layer, field, offset, bytes))
    return fail(TTTJ_ERR_INVALID, "no weight field %d at layer %d", field, layer);
  return TTTJ_OK;
}

size_t tttj_workspace_bytes(const tttj_config* cfg) {
  if (check_config(cfg)) return 0;
  return ws_layout(*cfg).total;
}

int tttj_device_sm_count(int device) { return sm_count(device); }

int tttj_path_choice(const tttj_config* cfg, int* fits, int* preferred, int* heads_per_step) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (!fits || !preferred || !heads_per_step) return fail(TTTJ_ERR_INVALID, "path_choice: null output");
  *fits = resident_fits(*cfg) ? 1 : 0;
  *preferred = (*fits && resident_preferred(*cfg)) ? 1 : 0;
  *heads_per_step = resident_gh(*cfg);
  return TTTJ_OK;
}

int tttj_gemm_tile(int rows, int n, int k, int epilogue, int num_sms, int* bn, int* pair) {
  static_assert(TTTJ_EPI_RESIDUAL_F32_STATS == EPI_RESIDUAL_F32_STATS &&
                    TTTJ_EPI_LN_FOLD == EPI_LN_FOLD && TTTJ_EPI_LN_FOLD_GELU == EPI_LN_FOLD_GELU &&
                    TTTJ_EPI_BIAS_RESIDUAL_F32 == EPI_BIAS_RESIDUAL_F32,
                "public and internal epilogue codes differ");
  if (!bn || !pair) return fail(TTTJ_ERR_INVALID, "gemm_tile: null output");
  if (rows < 0 || n <= 0 || k <= 0 || num_sms <= 0 || epilogue < 0 ||
      epilogue > TTTJ_EPI_LN_FOLD_GELU)
    return fail(TTTJ_ERR_INVALID, "gemm_tile: bad arguments");
  gemm_choose(rows, n, k, epilogue, num_sms, bn, pair);
  return TTTJ_OK;
}

size_t tttj_folded_bytes(const tttj_config* cfg) {
  if (check_config(cfg)) return 0;
  return folded_bytes(*cfg);
}

int tttj_fold_weights(const tttj_config* cfg, const void* weights, void* folded,
                      size_t folded_bytes_given, void* stream) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (!weights || !folded) return fail(TTTJ_ERR_INVALID, "fold_weights: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(weights) | reinterpret_cast<uintptr_t>(folded)) & (kAlign - 1))
    return fail(TTTJ_ERR_INVALID, "fold_weights: weights and folded must be 256-byte aligned");
  const size_t need = folded_bytes(*cfg);
  if (folded_bytes_given < need)
    return fail(TTTJ_ERR_INVALID, "fold_weights: buffer too small: %zu < %zu", folded_bytes_given,
                need);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int D = cfg->d_model, F = cfg->ffn_dim, hd = head_dim_of(*cfg), hp = layout_hd(*cfg);
  const int Q = (int)qkv_width(*cfg);
  const FoldLayout fl = fold_layout(*cfg);
  const uint8_t* wb = static_cast<const uint8_t*>(weights);
  auto W = [&](int layer, int field) -> const uint8_t* {
    size_t off = 0, bytes = 0;
    weight_offset(*cfg, layer, field, &off, &bytes);
    return wb + off;
  };
  for (int l = 0; l < cfg->num_layers; ++l) {
    uint8_t* fb = static_cast<uint8_t*>(folded) + (size_t)l * fl.total;
    // LN1 into the QKV weights (head-padded layout), LN2 into ffn_in.
    TTTJ_CUDA(fold_ln_launch(reinterpret_cast<const __half*>(W(l, TTTJ_W_QKV)),
                             reinterpret_cast<const float*>(W(l, TTTJ_B_QKV)),
                             reinterpret_cast<const float*>(W(l, TTTJ_LN1_W)),
                             reinterpret_cast<const float*>(W(l, TTTJ_LN1_B)), 3 * Q, D, hd, hp,
                             reinterpret_cast<__half*>(fb + fl.wqkv),
                             reinterpret_cast<float*>(fb + fl.bqkv),
                             reinterpret_cast<float*>(fb + fl.cqkv), s));
    TTTJ_CUDA(fold_ln_launch(reinterpret_cast<const __half*>(W(l, TTTJ_W_FFN_IN)),
                             reinterpret_cast<const float*>(W(l, TTTJ_B_FFN_IN)),
                             reinterpret_cast<const float*>(W(l, TTTJ_LN2_W)),
                             reinterpret_cast<const float*>(W(l, TTTJ_LN2_B)), F, D, 1, 1,
                             reinterpret_cast<__half*>(fb + fl.w1),
                             reinterpret_cast<float*>(fb + fl.b1),
                             reinterpret_cast<float*>(fb + fl.c1), s));
    if (heads_padded(*cfg))
      TTTJ_CUDA(pad_head_cols_launch(reinterpret_cast<const __half*>(W(l, TTTJ_W_OUT)), D, D, hd,
                                     hp, reinterpret_cast<__half*>(fb + fl.wo), s));
  }
  return TTTJ_OK;
}

}  // extern "C"

namespace {
// A rank's share of one sequence split across ranks (tttj_plan_create_cp).
struct CpArgs {
  int len;   // valid tokens of the sequence (positions 0 .. len - 1)
  int lo;    // first of this rank's rows
  int full;  // rows of the whole-sequence qkv / ctx buffers (>= len)
};

int plan_create_impl(const tttj_config* cfg, int device, const void* weights, const void* folded,
                     void* workspace, size_t workspace_bytes, const CpArgs* cp,
                     tttj_plan** out_plan) {
  int rc = check_config(cfg);
  if (rc) return rc;
  if (!weights || !folded || !workspace || !out_plan)
    return fail(TTTJ_ERR_INVALID, "null pointer argument");
  const WsLayout lay = ws_layout(*cfg, cp ? (size_t)cp->full : 0);
  if (workspace_bytes < lay.total)
    return fail(TTTJ_ERR_INVALID, "workspace too small: %zu < %zu", workspace_bytes, lay.total);
  if ((reinterpret_cast<uintptr_t>(weights) | reinterpret_cast<uintptr_t>(workspace) |
       reinterpret_cast<uintptr_t>(folded)) & (kAlign - 1))
    return fail(TTTJ_ERR_INVALID, "weights, folded weights and workspace must be 256-byte aligned");
  DeviceGuard guard(device);
  int cc_major = 0, cc_minor = 0;
  TTTJ_CUDA(cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, device));
  TTTJ_CUDA(cudaDeviceGetAttribute(&cc_minor, cudaDevAttrComputeCapabilityMinor, device));
  if (cc_major != 10 || cc_minor != 0)
    return fail(TTTJ_ERR_INVALID, "device %d is sm_%d%d; this library is built for sm_100a only",
                device, cc_major, cc_minor);

  tttj_plan* p = new tttj_plan();
  auto bail = [&](int code) {
    plan_release(p);
    delete p;
    return code;
  };
  p->cfg = *cfg;
  p->device = device;
  p->num_sms = sm_count(device);
  p->weights = static_cast<const uint8_t*>(weights);
  p->folded = static_cast<const uint8_t*>(folded);
  p->fold_layer = fold_layout(*cfg).total;
  p->ws = static_cast<uint8_t*>(workspace);
  p->lay = lay;
  p->tp = token_plan_at(p->ws, lay);
  if (cp) {
    p->cp = true;
    p->cp_lo = cp->lo;
    p->cp_len = cp->len;
    p->cp_full = cp->full;
    WsLayout wa{};
    plan_layout(1, cp->full, cfg->num_heads, &wa);
    p->tp_attn = token_plan_at(p->ws + lay.attn_plan, wa);
  }
  p->status = reinterpret_cast<int*>(p->ws + lay.status);
  p->resid = reinterpret_cast<float*>(p->ws + lay.resid);
  p->x16 = reinterpret_cast<__half*>(p->ws + lay.x16);
  p->stats = reinterpret_cast<float2*>(p->ws + lay.stats);
  p->pivot = reinterpret_cast<float*>(p->ws + lay.pivot);
  p->qkv = reinterpret_cast<__half*>(p->ws + lay.qkv);
  p->ctx = reinterpret_cast<__half*>(p->ws + lay.ctx);
  p->hid = reinterpret_cast<__half*>(p->ws + lay.hid);
  {
    void* h = nullptr;
    cudaError_t e = cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaHostAlloc(status mirror)"));
    p->status_host = static_cast<int*>(h);
    *reinterpret_cast<volatile int*>(p->status_host) = 0;
    e = cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming);
    if (e != cudaSuccess) return bail(cuda_fail(e, "cudaEventCreate(plan)"));
  }

  const int B = cfg->batch_size, S = cfg->seq_len, D = cfg->d_model, F = cfg->ffn_dim;
  const int T = B * S;
  const int* rows_dev = p->tp.seq_off + B;  // number of valid tokens
  // Statistics partials: two column halves per column tile of the residual GEMM that
  // writes them (out_proj -> LN2, ffn_out -> LN1), set once those GEMMs are built.
  // The gather writes layer 0's LN1 statistics as partial 0 (the rest zero), which
  // any count reads correctly.
  p->parts = 0;
  p->parts_ln2 = 0;
  const int hd = head_dim_of(*cfg), hp = layout_hd(*cfg), Q = (int)qkv_width(*cfg);
  auto W = [&](int layer, int field) -> const uint8_t* {
    size_t off = 0, bytes = 0;
    weight_offset(*cfg, layer, field, &off, &bytes);
    return p->weights + off;
  };
  p->layers.resize(cfg->num_layers);
  const FoldLayout fl = fold_layout(*cfg);
  // Two statistics buffers with their pivots, reused by every layer: ffn_out(l-1) /
  // the gather write LN1 for qkv(l); out_proj(l) writes LN2 for ffn_in(l).  Each
  // residual GEMM takes its pivot from the other buffer (the statistics of the
  // residual it adds to).
  float2* st_ln1 = p->stats;
  float2* st_ln2 = p->stats + (size_t)T * stats_parts(*cfg);
  float* pv_ln1 = p->pivot;
  float* pv_ln2 = p->pivot + T;
  for (int l = 0; l < cfg->num_layers; ++l) {
    LayerGemms& L = p->layers[l];
    L.ln1_w = reinterpret_cast<const float*>(W(l, TTTJ_LN1_W));
    L.ln1_b = reinterpret_cast<const float*>(W(l, TTTJ_LN1_B));
    L.ln2_w = reinterpret_cast<const float*>(W(l, TTTJ_LN2_W));
    L.ln2_b = reinterpret_cast<const float*>(W(l, TTTJ_LN2_B));
    const uint8_t* fb = p->folded + (size_t)l * p->fold_layer;
    const __half* wqkv_f = reinterpret_cast<const __half*>(fb + fl.wqkv);
    const __half* w1_f = reinterpret_cast<const __half*>(fb + fl.w1);
    const float* bqkv_f = reinterpret_cast<const float*>(fb + fl.bqkv);
    const float* cqkv = reinterpret_cast<const float*>(fb + fl.cqkv);
    const float* b1_f = reinterpret_cast<const float*>(fb + fl.b1);
    const float* c1 = reinterpret_cast<const float*>(fb + fl.c1);
    const __half* wo_pad = heads_padded(*cfg) ? reinterpret_cast<const __half*>(fb + fl.wo) : nullptr;
    if (l == 0) {
      // Tile widths of the residual GEMMs (the choice build_gemm makes below), which
      // fix the partial counts; every layer has the same shapes.
      int out_bn = 0, ffn_bn = 0, pair = 0;
      gemm_choose(T, D, Q, EPI_RESIDUAL_F32_STATS, p->num_sms, &out_bn, &pair);
      gemm_choose(T, D, F, EPI_RESIDUAL_F32_STATS, p->num_sms, &ffn_bn, &pair);
      p->parts_ln2 = 2 * ((D + out_bn - 1) / out_bn);
      p->parts = 2 * ((D + ffn_bn - 1) / ffn_bn);
    }
    // A split plan writes its rows' q|k|v at their sequence positions.
    __half* qkv_out = p->qkv + (cp ? (size_t)cp->lo * 3 * Q : 0);
    rc = build_gemm(&L.qkv, p->x16, D, wqkv_f, D, bqkv_f, qkv_out, 3 * Q, nullptr, 0, T, rows_dev,
                    3 * Q, D, EPI_LN_FOLD, p->status, p->num_sms);
    L.qkv.p.stats_in = st_ln1;
    L.qkv.p.stats_parts = p->parts;
    L.qkv.p.colsum = cqkv;
    L.qkv.p.ln_eps = kLnEps;
    if (!rc)
      rc = build_gemm(&L.out, p->ctx + (cp ? (size_t)cp->lo * Q : 0), Q,
                      wo_pad ? static_cast<const void*>(wo_pad) : W(l, TTTJ_W_OUT),
                      Q, reinterpret_cast<const float*>(W(l, TTTJ_B_OUT)), p->resid, D, p->resid,
                      D, T, rows_dev, D, Q, EPI_RESIDUAL_F32_STATS, p->status, p->num_sms);
    L.out.p.out16 = p->x16;
    L.out.p.ld16 = D;
    L.out.p.stats_out = st_ln2;
    L.out.p.stats_parts = p->parts_ln2;
    L.out.p.pivot_out = pv_ln2;
    L.out.p.stats_prev = st_ln1;
    L.out.p.pivot_prev = pv_ln1;
    L.out.p.stats_prev_parts = p->parts;
    if (!rc)
      rc = build_gemm(&L.ffn_in, p->x16, D, w1_f, D, b1_f, p->hid, F, nullptr, 0, T, rows_dev, F,
                      D, EPI_LN_FOLD_GELU, p->status, p->num_sms);
    L.ffn_in.p.stats_in = st_ln2;
    L.ffn_in.p.stats_parts = p->parts_ln2;
    L.ffn_in.p.colsum = c1;
    L.ffn_in.p.ln_eps = kLnEps;
    const bool last = l + 1 == cfg->num_layers;
    if (!rc)
      rc = build_gemm(&L.ffn_out, p->hid, F, W(l, TTTJ_W_FFN_OUT), F,
                      reinterpret_cast<const float*>(W(l, TTTJ_B_FFN_OUT)), p->resid, D, p->resid,
                      D, T, rows_dev, D, F, last ? EPI_BIAS_RESIDUAL_F32 : EPI_RESIDUAL_F32_STATS,
                      p->status, p->num_sms);
    if (!rc && (2 * ((D + L.out.bn - 1) / L.out.bn) != p->parts_ln2 ||
                2 * ((D + L.ffn_out.bn - 1) / L.ffn_out.bn) != p->parts))
      rc = fail(TTTJ_ERR_INVALID, "internal: residual GEMM tile width mismatch");
    if (!last) {
      L.ffn_out.p.out16 = p->x16;
      L.ffn_out.p.ld16 = D;
      L.ffn_out.p.stats_out = st_ln1;  // LN1 of layer l+1
      L.ffn_out.p.stats_parts = p->parts;
      L.ffn_out.p.pivot_out = pv_ln1;
      L.ffn_out.p.stats_prev = st_ln2;
      L.ffn_out.p.pivot_prev = pv_ln2;
      L.ffn_out.p.stats_prev_parts = p->parts_ln2;
    }
    if (rc) return bail(rc);
  }
  p->lnf_w = reinterpret_cast<const float*>(W(cfg->num_layers, TTTJ_LNF_W));
  p->lnf_b = reinterpret_cast<const float*>(W(cfg->num_layers, TTTJ_LNF_B));

  if (cp)
    rc = build_attention(&p->attn_tm, &p->attn, &p->attn_grid, p->qkv, p->ctx, cp->full, 1, cp->full,
                         cfg->num_heads, hd, hp, p->tp_attn, p->status, p->num_sms);
  else
    rc = build_attention(&p->attn_tm, &p->attn, &p->attn_grid, p->qkv, p->ctx, T, B, S,
                         cfg->num_heads, hd, hp, p->tp, p->status, p->num_sms);
  if (rc) return bail(rc);
  if (resident_fits(*cfg) && !cp) {
    rc = build_resident(p, fl);
    if (rc) return bail(rc);
  }
  *out_plan = p;
  return TTTJ_OK;
}
}  // namespace

extern "C" {

int tttj_plan_create(const tttj_config* cfg, int device, const void* weights, const void* folded,
                     void* workspace, size_t workspace_bytes, tttj_plan** out_plan) {
  return plan_create_impl(cfg, device, weights, folded, workspace, workspace_bytes, nullptr,
                          out_plan);
}

size_t tttj_workspace_bytes_cp(const tttj_config* cfg, int full_rows) {
  if (check_config(cfg) || full_rows <= 0) return 0;
  return ws_layout(*cfg, (size_t)full_rows).total;
}

int tttj_plan_create_cp(const tttj_config* cfg, int device, const void* weights, const void* folded,
                        int seq_len_valid, int row_lo, int full_rows, void* workspace,
                        size_t workspace_bytes, tttj_plan** out_plan) {
  int rc = check_config(cfg);
  if (rc) return rc;
  const int item = atc_item_rows(layout_hd(*cfg));
  const int rows = cfg->seq_len;  // this rank's rows
  if (cfg->batch_size != 1)
    return fail(TTTJ_ERR_INVALID, "plan_create_cp: batch_size must be 1 (one sequence per split)");
  if (row_lo < 0 || row_lo % item || rows <= 0 || row_lo + rows > seq_len_valid ||
      seq_len_valid > full_rows)
    return fail(TTTJ_ERR_INVALID,
                "plan_create_cp: rows [%d, %d) of %d valid tokens (buffers of %d rows): the first "
                "row must be a multiple of %d and the share inside the sequence",
                row_lo, row_lo + rows, seq_len_valid, full_rows, item);
  if (row_lo + rows != seq_len_valid && (row_lo + rows) % item)
    return fail(TTTJ_ERR_INVALID, "plan_create_cp: a share that ends before the sequence does "
                "must end on a multiple of %d rows", item);
  const CpArgs cp{seq_len_valid, row_lo, full_rows};
  return plan_create_impl(cfg, device, weights, folded, workspace, workspace_bytes, &cp, out_plan);
}

int tttj_plan_cp_qkv(tttj_plan* p, size_t* offset, size_t* row_bytes, int* full_rows) {
  if (!p || !offset || !row_bytes || !full_rows) return fail(TTTJ_ERR_INVALID, "cp_qkv: null argument");
  if (!p->cp) return fail(TTTJ_ERR_INVALID, "cp_qkv: not a split plan");
  *offset = p->lay.qkv;
  *row_bytes = 3 * qkv_width(p->cfg) * sizeof(__half);
  *full_rows = p->cp_full;
  return TTTJ_OK;
}

int tttj_plan_set_path(tttj_plan* p, int path) {
  if (!p) return fail(TTTJ_ERR_INVALID, "set_path: null plan");
  if (path != TTTJ_PATH_AUTO && path != TTTJ_PATH_LAYERWISE && path != TTTJ_PATH_RESIDENT)
    return fail(TTTJ_ERR_INVALID, "set_path: unknown path %d", path);
  if (path == TTTJ_PATH_RESIDENT && !p->res_ok)
    return fail(TTTJ_ERR_INVALID,
                "set_path: the resident kernel does not fit this shape (seq_len <= 128, "
                "d_model <= 128 or 256, layout head_dim 32/64/128, TMEM and shared memory)");
  p->path = path;
  return TTTJ_OK;
}

int tttj_plan_path(tttj_plan* p) { return p && use_resident(p) ? 1 : 0; }

int tttj_plan_destroy(tttj_plan* plan) {
  if (plan) {
    DeviceGuard guard(plan->device);
    plan_release(plan);
  }
  delete plan;
  return TTTJ_OK;
}

int tttj_plan_launch_count(tttj_plan* plan) {
  return plan ? launches_per_forward(plan) : 0;
}

int tttj_plan_enable_timing(tttj_plan* p, int enable) {
  if (!p) return fail(TTTJ_ERR_INVALID, "timing: null plan");
  DeviceGuard guard(p->device);
  if (enable && !p->timing) {
    const int n = max_launches(p->cfg);  // the largest forward of any path
    p->ev_start.resize(n);
    p->ev_stop.resize(n);
    p->ev_class.assign(n, 0);
    for (int i = 0; i < n; ++i) {
      TTTJ_CUDA(cudaEventCreate(&p->ev_start[i]));
      TTTJ_CUDA(cudaEventCreate(&p->ev_stop[i]));
    }
  } else if (!enable && p->timing) {
    int rc = collect_timing(p);
    destroy_events(p);
    if (rc) return rc;
  }
  p->timing = enable != 0;
  for (int i = 0; i < TTTJ_KCLASS_COUNT; ++i) {
    p->class_ms[i] = 0.0;
    p->class_launches[i] = 0;
  }
  return TTTJ_OK;
}

int tttj_plan_kernel_times(tttj_plan* p, double* total_ms, long* launches) {
  if (!p || !total_ms || !launches) return fail(TTTJ_ERR_INVALID, "timing: null argument");
  DeviceGuard guard(p->device);
  if (p->timing) {
    int rc = collect_timing(p);
    if (rc) return rc;
  }
  for (int i = 0; i < TTTJ_KCLASS_COUNT; ++i) {
    total_ms[i] = p->class_ms[i];
    launches[i] = p->class_launches[i];
  }
  return TTTJ_OK;
}

const char* tttj_kernel_class_name(int cls) {
  static const char* names[TTTJ_KCLASS_COUNT] = {
      "plan_tokens", "layernorm", "gemm_qkv", "attention", "gemm_out_proj",
      "gemm_ffn_in_gelu", "gemm_ffn_out", "final_layernorm_scatter", "resident_stack"};
  return (cls >= 0 && cls < TTTJ_KCLASS_COUNT) ? names[cls] : "";
}

}  // extern "C"

namespace {
// Stage capture of one sequence at one layer (tttj_forward_debug).  Buffer layout in
// floats: layernorm [S, D], q, k, v [S, D], scores [H, S, S], softmax [H, S, S],
// pv [S, D], output_projection [S, D], ffn [S, D], then two [S, D] scratch rows.
struct DebugCapture {
  int layer, sequence;
  float* buf;
};
size_t debug_floats(const tttj_config& c) {
  const size_t S = c.seq_len, D = c.d_model, H = c.num_heads;
  return 9 * S * D + 2 * H * S * S;
}
}  // namespace

static int forward_impl(tttj_plan* p, const void* x, int x_dtype, const uint8_t* valid_mask,
                        void* out, void* stream_ptr, const DebugCapture* dbg,
                        tttj_exchange_fn exchange = nullptr, void* user = nullptr);

extern "C" int tttj_forward(tttj_plan* p, const void* x, int x_dtype, const uint8_t* valid_mask,
                            void* out, void* stream_ptr) {
  if (p && p->cp) return fail(TTTJ_ERR_INVALID, "forward: a split plan runs with tttj_forward_cp");
  return forward_impl(p, x, x_dtype, valid_mask, out, stream_ptr, nullptr);
}

extern "C" int tttj_forward_cp(tttj_plan* p, const void* x, int x_dtype, void* out,
                               tttj_exchange_fn exchange, void* user, void* stream_ptr) {
  if (!p || !p->cp) return fail(TTTJ_ERR_INVALID, "forward_cp: not a split plan");
  if (!exchange) return fail(TTTJ_ERR_INVALID, "forward_cp: null exchange callback");
  return forward_impl(p, x, x_dtype, nullptr, out, stream_ptr, nullptr, exchange, user);
}

extern "C" size_t tttj_debug_floats(const tttj_config* cfg) {
  if (check_config(cfg)) return 0;
  return debug_floats(*cfg);
}

extern "C" int tttj_forward_debug(tttj_plan* p, const void* x, int x_dtype,
                                  const uint8_t* valid_mask, void* out, int layer, int sequence,
                                  float* debug, void* stream) {
  if (!p || !debug) return fail(TTTJ_ERR_INVALID, "forward_debug: null argument");
  if (p->cp) return fail(TTTJ_ERR_INVALID, "forward_debug: not available for split plans");
  if (layer < 0 || layer >= p->cfg.num_layers || sequence < 0 || sequence >= p->cfg.batch_size)
    return fail(TTTJ_ERR_INVALID, "forward_debug: layer %d / sequence %d out of range", layer,
                sequence);
  DebugCapture d{layer, sequence, debug};
  return forward_impl(p, x, x_dtype, valid_mask, out, stream, &d);
}

static int forward_impl(tttj_plan* p, const void* x, int x_dtype, const uint8_t* valid_mask,
                        void* out, void* stream_ptr, const DebugCapture* dbg,
                        tttj_exchange_fn exchange, void* user) {
  if (!p || !x || !out) return fail(TTTJ_ERR_INVALID, "forward: null argument");
  if (x_dtype != TTTJ_DTYPE_F16 && x_dtype != TTTJ_DTYPE_F32)
    return fail(TTTJ_ERR_INVALID, "forward: x must be fp16 or fp32");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 31)
    return fail(TTTJ_ERR_INVALID, "forward: x and out must be 32-byte aligned");
  DeviceGuard guard(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream_ptr);
  const tttj_config& c = p->cfg;
  const int B = c.batch_size, S = c.seq_len, D = c.d_model, T = B * S;
  const int hp = layout_hd(c);
  const int* rows_dev = p->tp.seq_off + B;

  // A bounded device wait of an earlier forward gave up (its last kernel copied the
  // status word into the pinned mirror): report it now, without synchronising, clear
  // it, and launch nothing.  The next call runs normally.
  {
    volatile int* mirror = p->status_host;
    const int v = mirror ? *mirror : 0;
    if (v != 0) {
      *mirror = 0;
      TTTJ_CUDA(cudaMemsetAsync(p->status, 0, sizeof(int), s));
      p->plan_static = false;
      return fail(TTTJ_ERR_DEVICE_TIMEOUT,
                  "a device wait of an earlier forward of this plan timed out (status 0x%x); "
                  "that forward's output is invalid",
                  v);
    }
  }
  // The workspace belongs to the plan: a forward on another stream than the previous
  // one first waits for the previous one.  A forward captured into a CUDA graph skips
  // this ordering (an event recorded outside the capture cannot be waited on inside
  // it): the capturing caller orders the capture after earlier work (torch.cuda.graph
  // synchronises the device first) and its replays after each other.
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  TTTJ_CUDA(cudaStreamIsCapturing(s, &capture));
  const bool capturing = capture != cudaStreamCaptureStatusNone;
  if (capturing && p->timing)
    return fail(TTTJ_ERR_INVALID, "forward: per-kernel timing cannot be on while the stream is capturing");
  if (!capturing && p->has_last && s != p->last_stream)
    TTTJ_CUDA(cudaStreamWaitEvent(s, p->done, 0));
  struct DoneRecord {  // record completion on every return path after launches began
    tttj_plan* p;
    cudaStream_t s;
    bool active;
    ~DoneRecord() {
      if (active && cudaEventRecord(p->done, s) == cudaSuccess) {
        p->last_stream = s;
        p->has_last = true;
      }
    }
  } done_record{p, s, !capturing};

  // Per-class timing: an event pair around every launch when enabled.
  if (p->timing) {
    int rc = collect_timing(p);
    if (rc) return rc;
  }
  size_t slot = 0;
  auto tick = [&](int cls) -> cudaError_t {
    if (!p->timing) return cudaSuccess;
    p->ev_class[slot] = cls;
    return cudaEventRecord(p->ev_start[slot], s);
  };
  auto tock = [&]() -> cudaError_t {
    if (!p->timing) return cudaSuccess;
    return cudaEventRecord(p->ev_stop[slot++], s);
  };
#define TTTJ_TIMED(cls, call)      \
  do {                             \
    TTTJ_CUDA(tick(cls));          \
    TTTJ_CUDA(call);               \
    TTTJ_CUDA(tock());             \
  } while (0)

  if (use_resident(p) && dbg == nullptr && !p->cp) {  // a capture always runs layer by layer
    // The whole stack in one launch: one CTA per sequence reads x and the mask directly.
    ResLaunch r = p->res;
    r.p.x = x;
    r.p.mask = valid_mask;
    r.p.out = out;
    r.p.x_f32 = x_dtype == TTTJ_DTYPE_F32 ? 1 : 0;
    TTTJ_TIMED(TTTJ_KCLASS_RESIDENT, resident_launch(r, s));
    p->ev_used = slot;
    return TTTJ_OK;
  }
  // Without a mask the plan is the all-valid one every time: built by the first such
  // forward, reused by the next ones (the reference caches the all-valid case too,
  // kernels/sequence_resident.py:173-192).
  // A captured forward always builds its plan, so that the graph does not depend on
  // what the forward before the capture left in the workspace; and once a plan has been
  // captured, its replays may rewrite the workspace's token plan behind the library's
  // back, so no later forward of it reuses one.
  if (capturing) p->captured = true;
  if (!(valid_mask == nullptr && p->plan_static) || p->captured) {
    TTTJ_TIMED(TTTJ_KCLASS_PLAN, plan_tokens_launch(valid_mask, B, S, c.num_heads, c.causal,
                                                    atc_item_rows(hp), ATC_BN, p->tp, s));
    // A split plan's attention: the whole sequence's keys, this rank's query blocks.
    if (p->cp)
      TTTJ_TIMED(TTTJ_KCLASS_PLAN,
                 plan_tokens_launch(nullptr, 1, p->cp_len, c.num_heads, c.causal,
                                    atc_item_rows(hp), ATC_BN, p->tp_attn, s, p->cp_lo,
                                    p->cp_lo + T));
  }
  p->plan_static = valid_mask == nullptr && !p->captured;
  const TokenPlan& tpa = p->cp ? p->tp_attn : p->tp;  // attention items and work counters
  TTTJ_TIMED(TTTJ_KCLASS_LAYERNORM,
             ln_gather_launch(x, x_dtype, p->tp.packed_src, rows_dev, T, D, p->resid, p->x16,
                              p->stats, p->pivot, p->parts, tpa.counters, s));
  // Capture buffers (floats) of tttj_forward_debug, filled at its layer.
  const size_t SD = (size_t)S * D, HSS = (size_t)c.num_heads * S * S;
  float* dg = dbg ? dbg->buf : nullptr;
  float *d_ln = dg, *d_q = dg + SD, *d_k = dg + 2 * SD, *d_v = dg + 3 * SD, *d_sc = dg + 4 * SD,
        *d_pr = d_sc + HSS, *d_pv = d_pr + HSS, *d_op = d_pv + SD, *d_ffn = d_op + SD,
        *d_x0 = d_ffn + SD, *d_x1 = d_x0 + SD;
  const int hd = head_dim_of(c), Qw = (int)qkv_width(c), bq = dbg ? dbg->sequence : 0;
  const int* dmap = p->tp.dst_map;
  for (int l = 0; l < c.num_layers; ++l) {
    // Every LayerNorm is folded into the GEMM that consumes it; the statistics come
    // from the gather (layer 0) or the preceding residual epilogue.
    const LayerGemms& L = p->layers[l];
    const bool cap = dbg && dbg->layer == l;
    if (cap) {  // block input x and its LN1 output
      TTTJ_CUDA(debug_gather_launch(p->resid, 0, D, 0, D, 1, 1, dmap, bq, S, d_x0, s));
      TTTJ_CUDA(debug_ln_launch(d_x0, L.ln1_w, L.ln1_b, kLnEps, S, D, dmap, bq, d_ln, s));
    }
    TTTJ_TIMED(TTTJ_KCLASS_GEMM_QKV, gemm_launch(L.qkv, s));
    if (cap) {
      TTTJ_CUDA(debug_gather_launch(p->qkv, 1, 3 * Qw, 0, D, hd, hp, dmap, bq, S, d_q, s));
      TTTJ_CUDA(debug_gather_launch(p->qkv, 1, 3 * Qw, Qw, D, hd, hp, dmap, bq, S, d_k, s));
      TTTJ_CUDA(debug_gather_launch(p->qkv, 1, 3 * Qw, 2 * Qw, D, hd, hp, dmap, bq, S, d_v, s));
      TTTJ_CUDA(debug_scores_launch(d_q, d_k, dmap, bq, S, c.num_heads, hd, c.causal,
                                    1.0f / sqrtf((float)hd), d_sc, d_pr, s));
    }
    if (p->cp) {
      // Every rank of the split has written its rows' q|k|v; the exchange (enqueued on
      // the stream by the caller) completes the whole sequence's before the attention.
      const int xr = exchange(user, l, stream_ptr);
      if (xr != 0) return fail(TTTJ_ERR_CUDA, "forward_cp: exchange failed at layer %d (%d)", l, xr);
    }
    AtcParams ap = p->attn;
    ap.work_counter = tpa.counters + l;
    TTTJ_TIMED(TTTJ_KCLASS_ATTENTION,
               attention_tc_launch(p->attn_tm, ap, hp, c.causal, p->attn_grid,
                                   p->cp ? p->cp_len : S, s));
    if (cap) TTTJ_CUDA(debug_gather_launch(p->ctx, 1, Qw, 0, D, hd, hp, dmap, bq, S, d_pv, s));
    TTTJ_TIMED(TTTJ_KCLASS_GEMM_OUT, gemm_launch(L.out, s));
    if (cap) {  // attention branch = x after the residual add - x before
      TTTJ_CUDA(debug_gather_launch(p->resid, 0, D, 0, D, 1, 1, dmap, bq, S, d_x1, s));
      TTTJ_CUDA(debug_diff_launch(d_x1, d_x0, (long)SD, d_op, s));
    }
    TTTJ_TIMED(TTTJ_KCLASS_GEMM_FFN_IN, gemm_launch(L.ffn_in, s));
    TTTJ_TIMED(TTTJ_KCLASS_GEMM_FFN_OUT, gemm_launch(L.ffn_out, s));
    if (cap) {  // FFN branch
      TTTJ_CUDA(debug_gather_launch(p->resid, 0, D, 0, D, 1, 1, dmap, bq, S, d_x0, s));
      TTTJ_CUDA(debug_diff_launch(d_x0, d_x1, (long)SD, d_ffn, s));
    }
  }
  TTTJ_TIMED(TTTJ_KCLASS_FINAL_LN,
             ln_final_launch(p->resid, p->tp.dst_map, T, D, p->lnf_w, p->lnf_b, kLnEps, out,
                             x_dtype, p->status, p->status_host, s));
#undef TTTJ_TIMED
  p->ev_used = slot;
  return TTTJ_OK;
}

extern "C" {

int tttj_plan_status(tttj_plan* p, int* device_status) {
  if (!p || !device_status) return fail(TTTJ_ERR_INVALID, "status: null argument");
  DeviceGuard guard(p->device);
  TTTJ_CUDA(cudaDeviceSynchronize());
  int v = 0;
  TTTJ_CUDA(cudaMemcpy(&v, p->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (v == 0 && p->status_host) v = *reinterpret_cast<volatile int*>(p->status_host);
  if (p->status_host) *reinterpret_cast<volatile int*>(p->status_host) = 0;
  if (v != 0) TTTJ_CUDA(cudaMemset(p->status, 0, sizeof(int)));
  if (v != 0) p->plan_static = false;  // a kernel gave up: rebuild the plan on the next forward
  *device_status = v;
  if (v != 0) return fail(TTTJ_ERR_DEVICE_TIMEOUT, "device wait timed out (status 0x%x)", v);
  return TTTJ_OK;
}

int tttj_linear(const void* a, int lda, const void* w, int ldw, const float* bias, void* out,
                int ldo, const void* residual, int ldr, int rows, const int* rows_dev, int n, int k,
                int epilogue, int* status_dev, void* stream) {
  if (!a || !w || !bias || !out) return fail(TTTJ_ERR_INVALID, "linear: null argument");
  if (epilogue < TTTJ_EPI_BIAS || epilogue > TTTJ_EPI_BIAS_RESIDUAL_F32)
    return fail(TTTJ_ERR_INVALID, "linear: unknown epilogue %d", epilogue);
  if (rows == 0) return TTTJ_OK;
  GemmLaunch g;
  int rc = build_gemm(&g, a, lda, w, ldw, bias, out, ldo, residual, ldr, rows, rows_dev, n, k,
                      epilogue, status_dev, -1);
  if (rc) return rc;
  TTTJ_CUDA(gemm_launch(g, static_cast<cudaStream_t>(stream)));
  return TTTJ_OK;
}

int tttj_layernorm(const void* in, void* out, int rows, int d, const float* gamma,
                   const float* beta, float eps, void* stream) {
  if (!in || !out || !gamma || !beta) return fail(TTTJ_ERR_INVALID, "layernorm: null argument");
  if (d <= 0 || d % 8 || d > 2048) return fail(TTTJ_ERR_INVALID, "layernorm: d=%d unsupported", d);
  if (rows < 0) return fail(TTTJ_ERR_INVALID, "layernorm: rows < 0");
  if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15)
    return fail(TTTJ_ERR_INVALID, "layernorm: pointers must be 16-byte aligned");
  TTTJ_CUDA(ln_rows_launch(in, 0, nullptr, rows, d, gamma, beta, eps,
                           static_cast<__half*>(out), static_cast<cudaStream_t>(stream)));
  return TTTJ_OK;
}

size_t tttj_attention_workspace_bytes(int batch, int seq_len, int num_heads) {
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0) return 0;
  WsLayout w{};
  return plan_layout(batch, seq_len, num_heads, &w);
}

int tttj_attention(const void* qkv, void* ctx, int qkv_rows, const uint8_t* valid_mask, int batch,
                   int seq_len, int d_model, int num_heads, int causal, void* workspace,
                   size_t workspace_bytes, void* stream) {
  if (!qkv || !ctx || !workspace) return fail(TTTJ_ERR_INVALID, "attention: null argument");
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0 || num_heads > 255 || d_model % num_heads ||
      qkv_rows <= 0)
    return fail(TTTJ_ERR_INVALID, "attention: bad shape");
  const int hd = d_model / num_heads;
  if (hd != 32 && hd != 64 && hd != 128 && hd != 256)
    return fail(TTTJ_ERR_INVALID, "attention: head_dim=%d unsupported (32, 64, 128, 256)", hd);
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(ctx)) & 15)
    return fail(TTTJ_ERR_INVALID, "attention: qkv and ctx must be 16-byte aligned");
  WsLayout w{};
  const size_t need = plan_layout(batch, seq_len, num_heads, &w);
  if (workspace_bytes < need)
    return fail(TTTJ_ERR_INVALID, "attention: workspace too small: %zu < %zu", workspace_bytes, need);
  int dev = 0;
  TTTJ_CUDA(cudaGetDevice(&dev));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  TokenPlan tp = token_plan_at(base, w);
  CUtensorMap tm;
  AtcParams ap;
  int grid = 0;
  int rc = build_attention(&tm, &ap, &grid, qkv, ctx, qkv_rows, batch, seq_len, num_heads, hd,
                           hd, tp, nullptr, sm_count(dev));
  if (rc) return rc;
  TTTJ_CUDA(plan_tokens_launch(valid_mask, batch, seq_len, num_heads, causal, atc_item_rows(hd),
                               ATC_BN, tp, s));
  TTTJ_CUDA(attention_tc_launch(tm, ap, hd, causal, grid, seq_len, s));
  return TTTJ_OK;
}

int tttj_selftest_wait_timeout(int* status_dev, uint64_t limit_ns, void* stream) {
  if (!status_dev) return fail(TTTJ_ERR_INVALID, "selftest: null status");
  TTTJ_CUDA(selftest_wait_launch(status_dev, nullptr, limit_ns, static_cast<cudaStream_t>(stream)));
  return TTTJ_OK;
}

int tttj_plan_selftest_timeout(tttj_plan* p, uint64_t limit_ns, void* stream) {
  if (!p) return fail(TTTJ_ERR_INVALID, "selftest: null plan");
  if (limit_ns > 1000000000ull) return fail(TTTJ_ERR_INVALID, "selftest: limit above 1 s");
  DeviceGuard guard(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->has_last && s != p->last_stream) TTTJ_CUDA(cudaStreamWaitEvent(s, p->done, 0));
  TTTJ_CUDA(selftest_wait_launch(p->status, p->status_host, limit_ns, s));
  TTTJ_CUDA(cudaEventRecord(p->done, s));
  p->last_stream = s;
  p->has_last = true;
  return TTTJ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free attention (tttj_attention_noalloc).
//
// Some callers cannot allocate device memory when they need attention: code that
// runs inside a memory-pool or allocator callback (re-entering the allocator would
// deadlock or recurse), hosts that forbid cudaMalloc once initialisation is over
// (cudaMalloc can synchronise the device and fail under a fixed memory budget),
// and runtimes that only hand a kernel its pre-placed input and output buffers.
// For them this entry point keeps the token plan and the attention work list in a
// fixed array of TTTJ_ATTENTION_NOALLOC_SCRATCH_BYTES that lives in the library's
// own device memory; every GPU that loads the library holds that array until the
// process exits.
//
// Host code must not pass g_attn_noalloc_scratch itself to a kernel: on the host the
// name is only a stand-in for the device symbol.  The device address is looked up with
// cudaGetSymbolAddress, with the device current, on the first call in each CUDA
// context (the first call on a device, and again after a device reset or in a new
// context: the cache is keyed by the context's process-unique id, so a stale address
// is never reused).  That first call may also make the CUDA runtime load the
// library's device code (lazy module loading), which allocates: it should come before
// any stream capture and outside any allocator or memory-pool callback.
//
// All calls on a device share the one array and it keeps whatever the last call
// wrote.  Nothing in it needs clearing: each call's plan kernel rewrites every value
// its attention kernel later reads.  Calls whose kernels overlap on the GPU (for
// example on two streams at once) race on the array and give wrong results.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoallocScratchBytes = TTTJ_ATTENTION_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kNoallocScratchBytes];

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
struct NoallocSlot {
  unsigned long long ctx_id = 0;  // 0: empty
  void* addr = nullptr;
};
NoallocSlot g_noalloc_slot[kNoallocMaxDevices];

// Process-unique id of the calling thread's current CUDA context (driver entry points
// cuCtxGetCurrent / cuCtxGetId), or 0 when it cannot be determined.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the scratch array on `device` (the current device).
int noalloc_scratch_address(int device, void** out) {
  if (device < 0 || device >= kNoallocMaxDevices)
    return fail(TTTJ_ERR_INVALID, "attention_noalloc: device %d out of range", device);
  const unsigned long long ctx_id = current_context_id();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoallocSlot& slot = g_noalloc_slot[device];
  if (ctx_id == 0 || slot.ctx_id != ctx_id || slot.addr == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(attention scratch)");
    if (p == nullptr) return fail(TTTJ_ERR_CUDA, "attention_noalloc: null scratch address");
    slot.ctx_id = ctx_id;  // 0 (id unknown): looked up again on every call
    slot.addr = p;
  }
  *out = slot.addr;
  return TTTJ_OK;
}

}  // namespace

extern "C" int tttj_attention_noalloc(const void* qkv, void* ctx, int qkv_rows,
                                      const uint8_t* valid_mask, int batch, int seq_len,
                                      int d_model, int num_heads, int causal, void* stream) {
  if (!qkv || !ctx) return fail(TTTJ_ERR_INVALID, "attention_noalloc: null argument");
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0 || num_heads > 255 || d_model % num_heads ||
      qkv_rows <= 0)
    return fail(TTTJ_ERR_INVALID, "attention_noalloc: bad shape");
  const int hd = d_model / num_heads;
  if (hd != 32 && hd != 64 && hd != 128 && hd != 256)
    return fail(TTTJ_ERR_INVALID, "attention_noalloc: head_dim=%d unsupported (32, 64, 128, 256)",
                hd);
  if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(ctx)) & 15)
    return fail(TTTJ_ERR_INVALID, "attention_noalloc: qkv and ctx must be 16-byte aligned");
  WsLayout w{};
  const size_t need = plan_layout(batch, seq_len, num_heads, &w);
  if (need > kNoallocScratchBytes)
    return fail(TTTJ_ERR_INVALID,
                "attention_noalloc: batch=%d seq_len=%d num_heads=%d needs %zu bytes of scratch, "
                "more than the built-in %zu; use tttj_attention with a caller workspace",
                batch, seq_len, num_heads, need, kNoallocScratchBytes);
  int dev = 0;
  TTTJ_CUDA(cudaGetDevice(&dev));
  void* scratch = nullptr;
  int rc = noalloc_scratch_address(dev, &scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TokenPlan tp = token_plan_at(static_cast<uint8_t*>(scratch), w);
  CUtensorMap tm;
  AtcParams ap;
  int grid = 0;
  rc = build_attention(&tm, &ap, &grid, qkv, ctx, qkv_rows, batch, seq_len, num_heads, hd, hd,
                       tp, nullptr, sm_count(dev));
  if (rc) return rc;
  TTTJ_CUDA(plan_tokens_launch(valid_mask, batch, seq_len, num_heads, causal, atc_item_rows(hd),
                               ATC_BN, tp, s));
  TTTJ_CUDA(attention_tc_launch(tm, ap, hd, causal, grid, seq_len, s));
  return TTTJ_OK;
}
