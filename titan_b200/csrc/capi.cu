// C ABI (include/titan_moe.h): argument checks, workspace carving and the
// launch sequence of each entry point.  No entry point allocates device
// memory or synchronises the host; errors come back as status codes with a
// per-thread message.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/titan_moe.h"
#include "tmoe_internal.h"

using namespace tmoe;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TMOE_OK;
  return fail(TMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

thread_local tmoe_stage_fn g_hook = nullptr;
thread_local void* g_hook_ctx = nullptr;

inline void stage(const char* name) {
  if (g_hook) g_hook(g_hook_ctx, name);
}

#define TMOE_TRY(expr, what)                                   \
  do {                                                         \
    stage(what);                                               \
    int _rc = cuda_status((expr), what);                       \
    if (_rc != TMOE_OK) return _rc;                            \
  } while (0)

// Carves 256-byte aligned pieces out of the caller's workspace.  With a null
// base it only measures.
struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

// tiles of `tile` rows over R sorted rows of E experts (a bound: one partial tile per expert)
int tiles_for(int R, int E, int tile) { return (R + tile - 1) / tile + E; }
// workspace capacity: enough for the smaller (swap-AB kernel) tile
int max_tiles(int R, int E) { return tiles_for(R, E, kSwTileN); }

bool bad_k(int K) { return K <= 0 || K % 64 != 0; }

}  // namespace

int tmoe::record_error(int code, const char* msg) { return fail(code, "%s", msg); }

extern "C" {

int tmoe_abi_version(void) { return TMOE_ABI_VERSION; }

void tmoe_set_stage_hook(tmoe_stage_fn fn, void* ctx) {
  g_hook = fn;
  g_hook_ctx = ctx;
}

int tmoe_device_status(void) {
  cudaDeviceSynchronize();
  const int tc = tc05_error_flag();
  if (tc == 2)
    return fail(TMOE_ERR_UNSUPPORTED,
                "the per-group tcgen05 kernel's bf16-activation path met a scale or activation "
                "outside fp16's exact range; prepare the layer's row normalisers "
                "(tmoe_prepare_row_scale) so that the swap-AB kernel runs it");
  if (tc || sw_error_flag())
    return fail(TMOE_ERR_TIMEOUT, "a tcgen05 kernel's bounded wait timed out");
  if (ep_error_flag())
    return fail(TMOE_ERR_TIMEOUT, "an expert-parallel exchange wait timed out");
  const int le = layer_error_flag();
  if (le == 2 || decode_range_flag())
    return fail(TMOE_ERR_UNSUPPORTED,
                "a decode-path activation group lay outside fp16's exact range (|x| >= 65504, "
                "or the whole group below 2^-14); run such tokens through the grouped-GEMM "
                "path (options.min_tokens <= T), which normalises x by a power of two");
  if (le)
    return fail(TMOE_ERR_TIMEOUT, "a grid barrier of the single-launch decode layer timed out");
  return TMOE_OK;
}

const char* tmoe_last_error(void) { return g_err.c_str(); }

// ---------------------------------------------------------------- weight prep

int tmoe_affine_quantize(const float* w, int64_t rows, int K, uint32_t* wq, uint16_t* scales,
                         uint16_t* biases, void* stream) {
  if (!w || !wq || !scales || !biases || rows < 0 || bad_k(K))
    return fail(TMOE_ERR_INVALID, "tmoe_affine_quantize: bad arguments (rows=%lld K=%d)",
                (long long)rows, K);
  TMOE_TRY(launch_affine_quantize(w, rows, K, wq, scales, biases, S(stream)), "affine_quantize");
  return TMOE_OK;
}

int tmoe_prepare_tables(const uint16_t* scales, const uint16_t* biases, int E, int N, int K,
                        uint16_t* scales_t, uint16_t* biases_t, void* stream) {
  if (!scales || !biases || !scales_t || !biases_t || E <= 0 || N <= 0 || bad_k(K))
    return fail(TMOE_ERR_INVALID, "tmoe_prepare_tables: bad arguments");
  TMOE_TRY(launch_prepare_tables(scales, biases, E, N, K / 64, scales_t, biases_t, S(stream)),
           "prepare_tables");
  return TMOE_OK;
}

int tmoe_prepare_row_scale(const uint16_t* scales, const uint16_t* biases, int E, int N, int K,
                           float* row_scale, void* stream) {
  if (!scales || !biases || !row_scale || E <= 0 || N <= 0 || bad_k(K))
    return fail(TMOE_ERR_INVALID, "tmoe_prepare_row_scale: bad arguments");
  TMOE_TRY(launch_row_scale(scales, biases, (long long)E * N, K, row_scale, S(stream)),
           "row_scale");
  return TMOE_OK;
}

int tmoe_qsum(const uint32_t* w, int E, int N, int K, uint16_t* qsum, void* stream) {
  if (!w || !qsum || E <= 0 || N <= 0 || bad_k(K))
    return fail(TMOE_ERR_INVALID, "tmoe_qsum: bad arguments");
  TMOE_TRY(launch_qsum(w, E, N, K, qsum, S(stream)), "qsum");
  return TMOE_OK;
}

int tmoe_quantize_activations(const uint16_t* x, int R, int K, int8_t* xq, float* xsc, float* xrs,
                              void* stream) {
  if (!x || !xq || !xsc || !xrs || R < 0 || bad_k(K))
    return fail(TMOE_ERR_INVALID, "tmoe_quantize_activations: bad arguments");
  TMOE_TRY(launch_quantize_rows(x, R, K, xq, xsc, xrs, S(stream)), "quantize_activations");
  return TMOE_OK;
}

// --------------------------------------------------------------------- router

static int check_router(int T, int H, int E, int k) {
  if (T < 0 || H <= 0 || H % 64 || E <= 0 || E > 1024 || k <= 0 || k > 32 || k > E)
    return fail(TMOE_ERR_UNSUPPORTED,
                "router: need H %% 64 == 0, 0 < E <= 1024, 0 < k <= min(32, E) (H=%d E=%d k=%d)",
                H, E, k);
  return TMOE_OK;
}

int tmoe_router_topk(const uint16_t* x, const uint16_t* router_w, int T, int H, int E, int k,
                     uint16_t* logits_ws, int32_t* idx, uint16_t* scores, uint16_t* probs_out,
                     void* stream) {
  if (!x || !router_w || !logits_ws || !idx || !scores)
    return fail(TMOE_ERR_INVALID, "tmoe_router_topk: null pointer");
  if (int rc = check_router(T, H, E, k)) return rc;
  if (T == 0) return TMOE_OK;
  TMOE_TRY(launch_router_logits(x, router_w, nullptr, T, H, E, logits_ws, nullptr, S(stream)),
           "router_logits");
  TMOE_TRY(launch_router_topk(logits_ws, T, E, k, idx, scores, probs_out, S(stream)), "router_topk");
  return TMOE_OK;
}

// -------------------------------------------------------------- routing plan

size_t tmoe_route_workspace_size(int R, int E) {
  if (R < 0 || E <= 0) return 0;
  return route_plan_scratch_bytes(R, E);
}

int tmoe_route_sort(const int32_t* idx, int R, int E, void* ws, size_t ws_bytes, int32_t* order,
                    int32_t* inv_order, int32_t* offsets, int32_t* tile_row, int32_t* tile_exp,
                    int32_t* ntiles, int maxt, void* stream) {
  if (!idx || !order || !inv_order || !offsets || R < 0 || E <= 0 || E > 1024)
    return fail(TMOE_ERR_INVALID, "tmoe_route_sort: bad arguments");
  if ((tile_row != nullptr) != (tile_exp != nullptr) || (tile_row && (!ntiles || maxt < 1)))
    return fail(TMOE_ERR_INVALID, "tmoe_route_sort: tile_row, tile_exp, ntiles and maxt go together");
  if (tile_row && maxt < tiles_for(R, E, kTileM))
    return fail(TMOE_ERR_INVALID, "tmoe_route_sort: maxt %d < ceil(R/128)+E = %d", maxt,
                tiles_for(R, E, kTileM));
  const size_t need = route_plan_scratch_bytes(R, E);
  if (need && (!ws || ws_bytes < need))
    return fail(TMOE_ERR_WORKSPACE, "tmoe_route_sort: workspace %zu < %zu bytes", ws_bytes, need);
  if (R == 0) return TMOE_OK;
  RoutePlan p{};
  p.order = order;
  p.inv = inv_order;
  p.offsets = offsets;
  p.tile_row = tile_row;
  p.tile_exp = tile_exp;
  p.ntiles = ntiles;
  TMOE_TRY(launch_route_plan(idx, R, E, kTileM, maxt, p, ws, S(stream)), "route_plan");
  return TMOE_OK;
}

// ------------------------------------------------------------------ gathers

namespace {

struct Int8GatherWs {
  int32_t *order, *inv, *offsets, *tile_row, *tile_exp, *ntiles;
  int8_t* xq;
  float *xsc, *xrs;
  void* route_scratch;
};

size_t carve_int8_gather(Carve& c, int R, int E, int K, Int8GatherWs* w) {
  const int maxt = max_tiles(R, E);
  Int8GatherWs t;
  t.order = c.take<int32_t>(R);
  t.inv = c.take<int32_t>(R);
  t.offsets = c.take<int32_t>(E + 1);
  t.tile_row = c.take<int32_t>(maxt);
  t.tile_exp = c.take<int32_t>(maxt);
  t.ntiles = c.take<int32_t>(1);
  t.xq = c.take<int8_t>((size_t)R * K * 2);     // fp16 codes of the tcgen05 operand layout
  t.xsc = c.take<float>((size_t)R * tc05_srow(K / 64));
  t.xrs = c.take<float>((size_t)R * tc05_srow(K / 64));
  t.route_scratch = c.take<uint8_t>(route_plan_scratch_bytes(R, E));
  if (w) *w = t;
  return c.off;
}

}  // namespace

size_t tmoe_gather_qmm_int8_workspace_size(int R, int E, int N, int K) {
  (void)N;
  if (R < 0 || E <= 0 || bad_k(K)) return 0;
  Carve c(nullptr);
  return carve_int8_gather(c, R, E, K, nullptr);
}

int tmoe_gather_qmm_int8(const uint16_t* x, const uint32_t* w, const uint16_t* scales_t,
                         const uint16_t* biases_t, const int32_t* rhs, int R, int E, int N, int K,
                         void* ws, size_t ws_bytes, uint16_t* y, void* stream) {
  if (!x || !w || !scales_t || !biases_t || !rhs || !y || R < 0 || E <= 0 || E > 1024)
    return fail(TMOE_ERR_INVALID, "tmoe_gather_qmm_int8: bad arguments");
  if (bad_k(K) || N <= 0 || N % 128)
    return fail(TMOE_ERR_UNSUPPORTED, "tmoe_gather_qmm_int8: need K %% 64 == 0 and N %% 128 == 0 (K=%d N=%d)", K, N);
  const size_t need = tmoe_gather_qmm_int8_workspace_size(R, E, N, K);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_gather_qmm_int8: workspace %zu < %zu bytes", ws_bytes, need);
  if (R == 0) return TMOE_OK;
  Carve c(ws);
  Int8GatherWs b;
  carve_int8_gather(c, R, E, K, &b);
  const int maxt = tiles_for(R, E, kTileM);
  RoutePlan p{};
  p.order = b.order;
  p.inv = b.inv;
  p.offsets = b.offsets;
  p.tile_row = b.tile_row;
  p.tile_exp = b.tile_exp;
  p.ntiles = b.ntiles;
  cudaStream_t s = S(stream);
  TMOE_TRY(launch_route_plan(rhs, R, E, kTileM, maxt, p, b.route_scratch, s), "route_plan");
  const bool tc = gemm_tc05_supported(K, N);
  GemmParams g{};
  if (tc) {
    // expert-sorted operand rows: row r quantises x row order[r]
    const int gs = tc05_srow(K / 64);
    TMOE_TRY(launch_prep_a16_rows(x, R, K, true, b.order, nullptr, 1, gs,
                                  reinterpret_cast<uint16_t*>(b.xq), b.xsc, b.xrs, s),
             "quantize_rows");
    g.A = b.xq;
    g.s_r = gs;
    g.a_nrows = R;
  } else {
    TMOE_TRY(launch_quantize_rows(x, R, K, b.xq, b.xsc, b.xrs, s), "quantize_rows");
    g.A = b.xq;
    g.s_r = K / 64;
    g.a_rows = b.order;
    g.a_div = 1;
  }
  g.asc = b.xsc;
  g.ars = b.xrs;
  g.s_g = 1;
  g.W = w;
  g.E = E;
  g.st = scales_t;
  g.bt = biases_t;
  g.tile_row = b.tile_row;
  g.tile_exp = b.tile_exp;
  g.ntiles = b.ntiles;
  g.offsets = b.offsets;
  g.K = K;
  g.N = N;
  g.Y = y;
  g.y_rows = b.order;
  // the per-group tcgen05 kernel (mma.sync for K > 3072 or N % 128 != 0): the
  // overlay's int8 algebra bit for bit
  if (tc)
    TMOE_TRY(launch_gemm_tc05(true, kEpiStore, g, maxt, s), "gemm_int8");
  else
    TMOE_TRY(launch_gemm_grouped(true, kEpiStore, g, maxt, s), "gemm_int8");
  return TMOE_OK;
}

namespace {

constexpr int kGemvMaxRows = 256;

struct Bf16GatherWs {
  int32_t *order, *inv, *offsets, *tile_row, *tile_exp, *ntiles, *uexp, *ustart, *nuniq;
  uint16_t* x16p;
  float* xsum;
  void* route_scratch;
  float* rs;        // swap-AB kernel: row normalisers, the x operand and its group scalars
  uint16_t* xb;
  float *xc1, *xc2;
};

size_t carve_bf16_gather(Carve& c, int R, int E, int N, int K, Bf16GatherWs* w) {
  const int maxt = max_tiles(R, E);
  const int U = R < E ? R : E;
  Bf16GatherWs t;
  t.order = c.take<int32_t>(R);
  t.inv = c.take<int32_t>(R);
  t.offsets = c.take<int32_t>(E + 1);
  t.tile_row = c.take<int32_t>(maxt);
  t.tile_exp = c.take<int32_t>(maxt);
  t.ntiles = c.take<int32_t>(1);
  t.uexp = c.take<int32_t>(U > 0 ? U : 1);
  t.ustart = c.take<int32_t>(U + 1);
  t.nuniq = c.take<int32_t>(1);
  t.x16p = c.take<uint16_t>((size_t)R * K);
  t.xsum = c.take<float>((size_t)R * (K / 64));
  t.route_scratch = c.take<uint8_t>(route_plan_scratch_bytes(R, E));
  t.rs = c.take<float>((size_t)E * N);
  t.xb = c.take<uint16_t>((size_t)R * K);
  t.xc1 = c.take<float>((size_t)R * (K / 64));
  t.xc2 = c.take<float>((size_t)R * (K / 64));
  if (w) *w = t;
  return c.off;
}

}  // namespace

size_t tmoe_gather_qmm_bf16_workspace_size(int R, int E, int N, int K) {
  if (R < 0 || E <= 0 || N <= 0 || bad_k(K)) return 0;
  Carve c(nullptr);
  return carve_bf16_gather(c, R, E, N, K, nullptr);
}

int tmoe_gather_qmm_bf16(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                         const uint16_t* biases, const uint16_t* scales_t,
                         const uint16_t* biases_t, const int32_t* rhs, int R, int E, int N, int K,
                         void* ws, size_t ws_bytes, uint16_t* y, void* stream) {
  if (!x || !w || !scales || !biases || !rhs || !y || R < 0 || E <= 0 || E > 1024)
    return fail(TMOE_ERR_INVALID, "tmoe_gather_qmm_bf16: bad arguments");
  if (bad_k(K) || N <= 0 || N % 128)
    return fail(TMOE_ERR_UNSUPPORTED, "tmoe_gather_qmm_bf16: need K %% 64 == 0 and N %% 128 == 0 (K=%d N=%d)", K, N);
  const bool gemv = R <= kGemvMaxRows;
  if (!gemv && (!scales_t || !biases_t))
    return fail(TMOE_ERR_INVALID, "tmoe_gather_qmm_bf16: R=%d > %d needs the prepared tables", R,
                kGemvMaxRows);
  const size_t need = tmoe_gather_qmm_bf16_workspace_size(R, E, N, K);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_gather_qmm_bf16: workspace %zu < %zu bytes", ws_bytes, need);
  if (R == 0) return TMOE_OK;
  Carve c(ws);
  Bf16GatherWs b;
  carve_bf16_gather(c, R, E, N, K, &b);
  cudaStream_t s = S(stream);
  const bool sw = !gemv && gemm_sw_supported(kEpiStore, K, N);
  const int tile = sw ? kSwTileN : kTileM;
  const int maxt = tiles_for(R, E, tile);
  const int U = R < E ? R : E;
  RoutePlan p{};
  p.order = b.order;
  p.inv = b.inv;
  p.offsets = b.offsets;
  if (gemv) {
    p.uexp = b.uexp;
    p.ustart = b.ustart;
    p.nuniq = b.nuniq;
  } else {
    p.tile_row = b.tile_row;
    p.tile_exp = b.tile_exp;
    p.ntiles = b.ntiles;
  }
  TMOE_TRY(launch_route_plan(rhs, R, E, tile, maxt, p, b.route_scratch, s), "route_plan");
  const int G = K / 64;
  if (gemv) {
    StreamParams q{};
    q.x = x;
    q.K = K;
    q.W = w;
    q.S = scales;
    q.B = biases;
    q.N = N;
    q.uexp = b.uexp;
    q.ustart = b.ustart;
    q.nuniq = b.nuniq;
    q.order = b.order;
    q.umax = U;
    q.col_div = 1;
    q.outb = y;
    TMOE_TRY(launch_gemv_stream(2, q, R, s), "gemv");
  } else if (sw) {
    // the swap-AB tcgen05 kernel, the row normalisers computed for this call
    TMOE_TRY(launch_row_scale(scales, biases, (long long)E * N, K, b.rs, s), "row_scale");
    TMOE_TRY(launch_prep_rows(x, R, K, false, b.xb, b.xc1, b.xc2, nullptr, s), "prep_x");
    SwParams g{};
    g.B = b.xb;
    g.c1 = b.xc1;
    g.c2 = b.xc2;
    g.b_rows = b.order;
    g.b_div = 1;
    g.W = w;
    g.st = scales_t;
    g.bt = biases_t;
    g.rscale = b.rs;
    g.E = E;
    g.K = K;
    g.Nw = N;
    g.tile_row = b.tile_row;
    g.tile_exp = b.tile_exp;
    g.ntiles = b.ntiles;
    g.offsets = b.offsets;
    g.maxt = maxt;
    g.Y = y;
    g.y_rows = b.order;
    TMOE_TRY(launch_gemm_sw(kEpiStore, g, s), "gemm_f16");
  } else {
    TMOE_TRY(launch_prep_x(x, R, K, b.x16p, b.xsum, G, 1, s), "prep_x");
    GemmParams g{};
    g.A = b.x16p;
    g.ars = b.xsum;
    g.s_r = G;
    g.s_g = 1;
    g.a_rows = b.order;
    g.a_div = 1;
    g.W = w;
    g.E = E;
    g.st = scales_t;
    g.bt = biases_t;
    g.tile_row = b.tile_row;
    g.tile_exp = b.tile_exp;
    g.ntiles = b.ntiles;
    g.offsets = b.offsets;
    g.K = K;
    g.N = N;
    g.Y = y;
    g.y_rows = b.order;
    TMOE_TRY(launch_gemm_grouped(false, kEpiStore, g, maxt, s), "gemm_f16");
  }
  return TMOE_OK;
}

// -------------------------------------------------------- decode-fused ops

namespace {

struct DecodeOpWs {
  int32_t *order, *inv, *offsets, *uexp, *ustart, *nuniq, *counters;
  uint16_t* a16;
  float* asum;
  float* part;
  void* route_scratch;
};

size_t carve_decode_op(Carve& c, int T, int k, int E, int K, int I, int D, DecodeOpWs* w) {
  const int R = T * k;
  const int U = R < E ? R : E;
  DecodeOpWs t;
  t.order = c.take<int32_t>(R);
  t.inv = c.take<int32_t>(R);
  t.offsets = c.take<int32_t>(E + 1);
  t.uexp = c.take<int32_t>(U > 0 ? U : 1);
  t.ustart = c.take<int32_t>(U + 1);
  t.nuniq = c.take<int32_t>(1);
  t.counters = c.take<int32_t>((D > 0 ? D : 32) / 32 + 1);
  t.a16 = c.take<uint16_t>((size_t)T * K);
  t.asum = c.take<float>((size_t)T * (K / 64));
  t.part = c.take<float>((size_t)R * (D > 0 ? D : 1));
  t.route_scratch = c.take<uint8_t>(route_plan_scratch_bytes(R, E));
  (void)I;
  if (w) *w = t;
  return c.off;
}

}  // namespace

size_t tmoe_decode_workspace_size(int T, int k, int E, int K, int I) {
  if (T < 0 || k <= 0 || E <= 0 || bad_k(K) || bad_k(I)) return 0;
  Carve c(nullptr);
  // down_wsum needs part [R, D]; D = K of the gate_up call (hidden size).
  return carve_decode_op(c, T, k, E, K, I, K, nullptr);
}

int tmoe_gate_up_silu(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                      const uint16_t* biases, const int32_t* idx, int T, int k, int E, int K, int I,
                      void* ws, size_t ws_bytes, float* h, void* stream) {
  if (!x || !w || !scales || !biases || !idx || !h || T < 0 || k <= 0 || E <= 0 || E > 1024)
    return fail(TMOE_ERR_INVALID, "tmoe_gate_up_silu: bad arguments");
  if (bad_k(K) || I <= 0 || I % 32)
    return fail(TMOE_ERR_UNSUPPORTED, "tmoe_gate_up_silu: need K %% 64 == 0, I %% 32 == 0");
  const size_t need = tmoe_decode_workspace_size(T, k, E, K, I);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_gate_up_silu: workspace %zu < %zu bytes", ws_bytes, need);
  if (T == 0) return TMOE_OK;
  Carve c(ws);
  DecodeOpWs b;
  carve_decode_op(c, T, k, E, K, I, K, &b);
  cudaStream_t s = S(stream);
  const int R = T * k, U = R < E ? R : E;
  RoutePlan p{};
  p.order = b.order;
  p.inv = b.inv;
  p.offsets = b.offsets;
  p.uexp = b.uexp;
  p.ustart = b.ustart;
  p.nuniq = b.nuniq;
  TMOE_TRY(launch_route_plan(idx, R, E, kTileM, 1, p, b.route_scratch, s), "route_plan");
  StreamParams q{};
  q.x = x;
  q.K = K;
  q.W = w;
  q.S = scales;
  q.B = biases;
  q.N = 2 * I;
  q.uexp = b.uexp;
  q.ustart = b.ustart;
  q.nuniq = b.nuniq;
  q.order = b.order;
  q.umax = U;
  q.col_div = k;
  q.out = h;
  TMOE_TRY(launch_gemv_stream(0, q, T, s), "gemv_gate_up");
  return TMOE_OK;
}

int tmoe_down_wsum(const float* h, const uint32_t* w, const uint16_t* scales,
                   const uint16_t* biases, const int32_t* idx, const float* scores, int T, int k,
                   int E, int I, int D, void* ws, size_t ws_bytes, uint16_t* y, void* stream) {
  if (!h || !w || !scales || !biases || !idx || !scores || !y || T < 0 || k <= 0 || E <= 0 ||
      E > 1024)
    return fail(TMOE_ERR_INVALID, "tmoe_down_wsum: bad arguments");
  if (bad_k(I) || D <= 0 || D % 64)
    return fail(TMOE_ERR_UNSUPPORTED, "tmoe_down_wsum: need I %% 64 == 0, D %% 64 == 0");
  Carve m(nullptr);
  const size_t need = carve_decode_op(m, T, k, E, D, I, D, nullptr);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_down_wsum: workspace %zu < %zu bytes", ws_bytes, need);
  if (T == 0) return TMOE_OK;
  Carve c(ws);
  DecodeOpWs b;
  carve_decode_op(c, T, k, E, D, I, D, &b);
  cudaStream_t s = S(stream);
  const int R = T * k, U = R < E ? R : E;
  RoutePlan p{};
  p.order = b.order;
  p.inv = b.inv;
  p.offsets = b.offsets;
  p.uexp = b.uexp;
  p.ustart = b.ustart;
  p.nuniq = b.nuniq;
  TMOE_TRY(launch_route_plan(idx, R, E, kTileM, 1, p, b.route_scratch, s), "route_plan");
  TMOE_TRY(launch_zero_i32(b.counters, D / 32, s), "zero_counters");
  StreamParams q{};
  q.h = h;
  q.K = I;
  q.W = w;
  q.S = scales;
  q.B = biases;
  q.N = D;
  q.uexp = b.uexp;
  q.ustart = b.ustart;
  q.nuniq = b.nuniq;
  q.order = b.order;
  q.umax = U;
  q.col_div = 1;
  q.out = b.part;
  q.counters = b.counters;
  q.scores_f32 = scores;
  q.T = T;
  q.k = k;
  q.y = y;
  TMOE_TRY(launch_gemv_stream(1, q, T, s), "gemv_down");
  return TMOE_OK;
}

// ---------------------------------------------------------------------- SwiGLU

int tmoe_swiglu(const uint16_t* gate_up, int R, int I, uint16_t* h, void* stream) {
  if (!gate_up || !h || R < 0 || I <= 0) return fail(TMOE_ERR_INVALID, "tmoe_swiglu: bad arguments");
  TMOE_TRY(launch_swiglu(gate_up, R, I, h, S(stream)), "swiglu");
  return TMOE_OK;
}

// --------------------------------------------------------------- weighted sum

int tmoe_weighted_sum(const uint16_t* ys, const int32_t* inv_order, const uint16_t* scores, int T,
                      int k, int D, int mode, uint16_t* out, void* stream) {
  if (!ys || !scores || !out || T < 0 || k <= 0 || (mode != 0 && mode != 1))
    return fail(TMOE_ERR_INVALID, "tmoe_weighted_sum: bad arguments");
  if (D <= 0 || D % 8) return fail(TMOE_ERR_UNSUPPORTED, "tmoe_weighted_sum: need D %% 8 == 0");
  TMOE_TRY(launch_wsum(ys, inv_order, scores, T, k, D, mode, nullptr, nullptr, out, S(stream)),
           "weighted_sum");
  return TMOE_OK;
}

// ------------------------------------------------ swap-AB expert GEMMs
// gate_up with the fused SwiGLU, then down, on gemm_sw: the activations and
// h quantised once each (prep_rows), the weights widened in shared memory.

namespace {

struct FastProj {                    // one expert projection pair
  const uint32_t* guw;
  const uint16_t *gust, *gubt;
  const float* gurs;
  const uint32_t* dnw;
  const uint16_t *dnst, *dnbt;
  const float* dnrs;
  int E, H, I;                       // gate_up [E][2I][H], down [E][H][I]
};

bool fast_ok(const FastProj& f) {
  return f.gurs && f.dnrs && f.gust && f.gubt && f.dnst && f.dnbt &&
         gemm_sw_supported(kEpiSwigluH16, f.H, 2 * f.I) && gemm_sw_supported(kEpiStore, f.I, f.H);
}

FastProj routed_proj(const tmoe_layer* L) {
  return {L->gate_up_w, L->gate_up_st, L->gate_up_bt, L->gate_up_rs,
          L->down_w,    L->down_st,    L->down_bt,    L->down_rs,
          L->num_experts, L->hidden, L->moe_inter};
}

FastProj shared_proj(const tmoe_layer* L) {
  return {L->shared_gate_up_w, L->shared_gate_up_st, L->shared_gate_up_bt, L->shared_gate_up_rs,
          L->shared_down_w,    L->shared_down_st,    L->shared_down_bt,    L->shared_down_rs,
          1, L->hidden, L->shared_inter};
}

struct FastWs {
  uint16_t* xb;        // activation operand rows [xrows][H] (codes, or x * 2^-Et)
  float *xc1, *xc2;    // [xrows][H/64]: group scale (or 2^Et) and exact group sum
  uint16_t* h;         // bf16 h [P][I], sorted rows
  uint16_t* hb;        // h operand rows [P][I]
  float *hc1, *hc2;    // [P][I/64]
};

void carve_fast(Carve& c, int xrows, int P, int H, int I, FastWs* w) {
  FastWs t;
  t.xb = c.take<uint16_t>((size_t)xrows * H);
  t.xc1 = c.take<float>((size_t)xrows * (H / 64));
  t.xc2 = c.take<float>((size_t)xrows * (H / 64));
  t.h = c.take<uint16_t>((size_t)P * I);
  t.hb = c.take<uint16_t>((size_t)P * I);
  t.hc1 = c.take<float>((size_t)P * (I / 64));
  t.hc2 = c.take<float>((size_t)P * (I / 64));
  if (w) *w = t;
}

struct FastRoute {                   // routed rows in expert order (route plan tiles of kSwTileN)
  const int32_t *tile_row, *tile_exp, *ntiles, *offsets;
  int maxt;
  const int32_t* b_rows;             // gate_up activation row of sorted row r:
  int b_div;                         //   b_rows[r] / b_div, or b_map[b_rows[r]]
  const int32_t* b_map;
};

// names: fold of x, gate_up GEMM, fold of h, down GEMM (stage-hook labels).
int run_fast(const FastProj& f, const uint16_t* x, int xrows, int prows, bool q_gu, bool q_dn,
             const FastRoute& rt, const FastWs& w, uint16_t* Y, const int32_t* y_rows,
             uint16_t* const* y_ptr, cudaStream_t s, const char* const names[4]) {
  TMOE_TRY(launch_prep_rows(x, xrows, f.H, q_gu, w.xb, w.xc1, w.xc2, nullptr, s), names[0]);
  SwParams g{};
  g.B = w.xb;
  g.c1 = w.xc1;
  g.c2 = w.xc2;
  g.b_rows = rt.b_rows;
  g.b_div = rt.b_div > 0 ? rt.b_div : 1;
  g.b_map = rt.b_map;
  g.W = f.guw;
  g.st = f.gust;
  g.bt = f.gubt;
  g.rscale = f.gurs;
  g.E = f.E;
  g.K = f.H;
  g.Nw = 2 * f.I;
  g.bias_bf16 = q_gu ? 1 : 0;
  g.tile_row = rt.tile_row;
  g.tile_exp = rt.tile_exp;
  g.ntiles = rt.ntiles;
  g.offsets = rt.offsets;
  g.maxt = rt.maxt;
  g.H = w.h;
  TMOE_TRY(launch_gemm_sw(kEpiSwigluH16, g, s), names[1]);
  // rows past offsets[E] (skipped slots) were not written and are not read
  TMOE_TRY(launch_prep_rows(w.h, prows, f.I, q_dn, w.hb, w.hc1, w.hc2, rt.offsets + f.E, s),
           names[2]);
  SwParams d{};
  d.B = w.hb;
  d.c1 = w.hc1;
  d.c2 = w.hc2;
  d.W = f.dnw;
  d.st = f.dnst;
  d.bt = f.dnbt;
  d.rscale = f.dnrs;
  d.E = f.E;
  d.K = f.I;
  d.Nw = f.H;
  d.bias_bf16 = q_dn ? 1 : 0;
  d.tile_row = rt.tile_row;
  d.tile_exp = rt.tile_exp;
  d.ntiles = rt.ntiles;
  d.offsets = rt.offsets;
  d.maxt = rt.maxt;
  d.Y = Y;
  d.y_rows = y_rows;
  d.y_ptr = y_ptr;
  TMOE_TRY(launch_gemm_sw(kEpiStore, d, s), names[3]);
  return TMOE_OK;
}

const char* const kRoutedNames[4] = {"quantize_rows", "gemm_gate_up", "quantize_h", "gemm_down"};
const char* const kSharedNames[4] = {"prep_x", "gemm_shared_gate_up", "prep_h_shared",
                                     "gemm_shared_down"};

}  // namespace

// ---------------------------------------------------------------- whole block

namespace {

struct BlockWs {
  uint16_t* logits;
  float* gate_logit;
  int32_t* idx;
  uint16_t* scores;
  int32_t *order, *inv, *offsets, *tile_row, *tile_exp, *ntiles, *uexp, *ustart, *nuniq;
  void* route_scratch;
  // decode
  int32_t* epoch;              // single-launch decode layer: launch epoch (offset 0, every path)
  unsigned long long* gucnt;   // ... its gate_up-tiles-done counter (offset 256)
  // ... and its exchanges: epoch-tagged logits and gate logits, CTA start
  // marks, h of the routed pairs and of the shared expert
  unsigned long long *tlog, *tgate;
  int32_t* tseen;
  uint32_t *th, *ths;
  int32_t* counters;
  uint16_t* x16p;
  float *xsum, *h, *hs, *part, *part_sh;
  // prefill
  int8_t *xq, *hq;
  float *xsc, *xrs, *hsc, *hrs;
  uint16_t *h16p, *ys;
  int32_t *s_tile_row, *s_tile_exp, *s_ntiles, *s_offsets;
  uint16_t *sx16p, *sh16p, *ys_sh;  // sx16p/sxsum: fp16 operand copy of x (F16 GEMMs)
  float *sxsum, *shrs;
  FastWs fr, fs;                    // swap-AB path: routed experts, shared expert
};

int opt_min_tokens(const tmoe_options* o) { return (o && o->min_tokens > 0) ? o->min_tokens : 512; }
int opt_down_int8(const tmoe_options* o) { return o ? (o->down_int8 != 0) : 1; }
int opt_wsum(const tmoe_options* o) { return o ? o->wsum_mode : 0; }
int opt_int8(const tmoe_options* o) { return o ? (o->int8_prefill != 0) : 1; }
int opt_gemm(const tmoe_options* o) { return o ? o->gemm_kernel : 0; }
// the persistent tile tcgen05 kernel (else mma.sync) where the swap-AB one is not used
int opt_tc05(const tmoe_options* o) { return opt_gemm(o) != 1; }
// The per-group tcgen05 kernel runs every grouped GEMM of the layer when it is
// selected and takes all of the layer's shapes (K <= 3072, N % 128 == 0);
// otherwise the mma.sync kernel does.
bool tc05_layer(const tmoe_layer* L, const tmoe_options* o) {
  const int H = L->hidden, I = L->moe_inter, Is = L->shared_inter;
  return opt_tc05(o) && gemm_tc05_supported(H, 2 * I) && gemm_tc05_supported(I, H) &&
         (Is == 0 || (gemm_tc05_supported(H, 2 * Is) && gemm_tc05_supported(Is, H)));
}
// routed experts on the swap-AB kernel: when asked for (gemm_kernel 2), and
// for the stock (bf16-activation) semantics whenever the layer carries its
// row normalisers (the power-of-two normalisers keep x and the scales exact
// in fp16 at any magnitude)
bool fast_routed(const tmoe_layer* L, const tmoe_options* o) {
  return fast_ok(routed_proj(L)) && (opt_gemm(o) == 2 || !opt_int8(o));
}
bool fast_shared(const tmoe_layer* L) { return L->shared_inter > 0 && fast_ok(shared_proj(L)); }
int opt_layer(const tmoe_options* o) { return o ? (o->decode_kernel == 0) : 1; }

size_t carve_block(Carve& c, const tmoe_layer* L, int T, const tmoe_options* opt, BlockWs* out) {
  const int H = L->hidden, E = L->num_experts, k = L->top_k, I = L->moe_inter,
            Is = L->shared_inter;
  const int R = T * k, U = R < E ? R : E, G = H / 64;
  const bool prefill = T >= opt_min_tokens(opt);
  const int maxt = max_tiles(R, E);
  BlockWs b{};
  // The single-launch decode layer's epoch word and gate_up counter first, at
  // the same offsets for every path and shape (only that kernel writes them),
  // then the self-resetting counters: the decode router's ticket and one
  // combine counter per 32-row output slab.
  b.epoch = c.take<int32_t>(1);
  b.gucnt = c.take<unsigned long long>(1);
  b.counters = c.take<int32_t>(H / 32 + 1);
  b.logits = c.take<uint16_t>((size_t)T * E);
  b.gate_logit = c.take<float>(T > 0 ? T : 1);
  b.idx = c.take<int32_t>(R);
  b.scores = c.take<uint16_t>(R);
  b.order = c.take<int32_t>(R);
  b.inv = c.take<int32_t>(R);
  b.offsets = c.take<int32_t>(E + 1);
  b.route_scratch = c.take<uint8_t>(route_plan_scratch_bytes(R, E));
  if (!prefill) {
    if (T <= kLayerMaxT) {
      b.tlog = c.take<unsigned long long>((size_t)T * E);
      b.tgate = c.take<unsigned long long>(T);
      b.tseen = c.take<int32_t>(kLayerMaxCtas);
      b.th = c.take<uint32_t>((size_t)R * I);
      if (Is > 0) b.ths = c.take<uint32_t>((size_t)T * Is);
    }
    b.uexp = c.take<int32_t>(U > 0 ? U : 1);
    b.ustart = c.take<int32_t>(U + 1);
    b.nuniq = c.take<int32_t>(1);
    b.h = c.take<float>((size_t)R * I);
    b.part = c.take<float>((size_t)R * H);
    if (Is > 0) {
      b.hs = c.take<float>((size_t)T * Is);
      b.part_sh = c.take<float>((size_t)T * H);
    }
  } else {
    const bool i8 = opt_int8(opt), d8 = i8 && opt_down_int8(opt);
    b.tile_row = c.take<int32_t>(maxt);
    b.tile_exp = c.take<int32_t>(maxt);
    b.ntiles = c.take<int32_t>(1);
    const bool tc = tc05_layer(L, opt);
    const bool fr = fast_routed(L, opt), fs = fast_shared(L);
    const int gs = tc ? tc05_srow(G) : G, gi = tc ? tc05_srow(I / 64) : I / 64;
    if (fr) {
      carve_fast(c, T, R, H, I, &b.fr);
    } else {
      if (tc) {  // tcgen05: expert-sorted fp16 rows (int8 codes or x) + row scalars
        b.xq = c.take<int8_t>((size_t)R * H * 2);
        b.xsc = c.take<float>((size_t)R * gs);
        b.xrs = c.take<float>((size_t)R * gs);
      } else if (i8) {  // mma.sync: int8 codes per token
        b.xq = c.take<int8_t>((size_t)T * H);
        b.xsc = c.take<float>((size_t)T * G);
        b.xrs = c.take<float>((size_t)T * G);
      }
      if (d8) {
        if (tc)
          b.h16p = c.take<uint16_t>((size_t)R * I);
        else
          b.hq = c.take<int8_t>((size_t)R * I);
        b.hsc = c.take<float>((size_t)R * gi);
      } else {
        b.h16p = c.take<uint16_t>((size_t)R * I);
      }
      b.hrs = c.take<float>((size_t)R * gi);
    }
    if ((!fr && !i8 && !tc) || (Is > 0 && !fs)) {
      b.sx16p = c.take<uint16_t>((size_t)T * H);
      b.sxsum = c.take<float>((size_t)T * gs);
    }
    b.ys = c.take<uint16_t>((size_t)R * H);
    if (Is > 0) {
      const int st = (T + kSwTileN - 1) / kSwTileN;
      b.s_tile_row = c.take<int32_t>(st);
      b.s_tile_exp = c.take<int32_t>(st);
      b.s_ntiles = c.take<int32_t>(1);
      b.s_offsets = c.take<int32_t>(2);
      if (fs) {
        carve_fast(c, T, T, H, Is, &b.fs);
      } else {
        b.sh16p = c.take<uint16_t>((size_t)T * Is);
        b.shrs = c.take<float>((size_t)T * (tc ? tc05_srow(Is / 64) : Is / 64));
      }
      b.ys_sh = c.take<uint16_t>((size_t)T * H);
    }
  }
  if (out) *out = b;
  return c.off;
}

int check_layer(const tmoe_layer* L, int T, const tmoe_options* opt) {
  if (!L) return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: null layer");
  const int H = L->hidden, E = L->num_experts, k = L->top_k, I = L->moe_inter,
            Is = L->shared_inter;
  if (T < 0 || I <= 0 || Is < 0) return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: bad sizes");
  if (int rc = check_router(T, H, E, k)) return rc;
  if (!L->router_w || !L->gate_up_w || !L->gate_up_s || !L->gate_up_b || !L->down_w ||
      !L->down_s || !L->down_b)
    return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: missing routed weights");
  if (I % 64 || H % 128)
    return fail(TMOE_ERR_UNSUPPORTED, "tmoe_moe_forward: need I %% 64 == 0 and H %% 128 == 0 (H=%d I=%d)", H, I);
  if (Is > 0) {
    if (!L->shared_gate_up_w || !L->shared_gate_up_s || !L->shared_gate_up_b ||
        !L->shared_down_w || !L->shared_down_s || !L->shared_down_b || !L->shared_gate_w)
      return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: missing shared-expert weights");
    if (Is % 64) return fail(TMOE_ERR_UNSUPPORTED, "tmoe_moe_forward: need Is %% 64 == 0");
  }
  if (T >= opt_min_tokens(opt)) {
    if (!L->gate_up_st || !L->gate_up_bt || !L->down_st || !L->down_bt)
      return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: the int8 path needs the prepared tables");
    if (Is > 0 && (!L->shared_gate_up_st || !L->shared_gate_up_bt || !L->shared_down_st ||
                   !L->shared_down_bt))
      return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: the shared expert needs its prepared tables");
  }
  return TMOE_OK;
}

}  // namespace

size_t tmoe_moe_workspace_size(const tmoe_layer* L, int T, const tmoe_options* opt) {
  if (!L || T < 0) return 0;
  Carve c(nullptr);
  return carve_block(c, L, T, opt, nullptr);
}

int tmoe_moe_forward(const tmoe_layer* L, const uint16_t* x, int T, const tmoe_options* opt,
                     void* ws, size_t ws_bytes, uint16_t* y, int32_t* idx_out,
                     uint16_t* scores_out, void* stream) {
  if (int rc = check_layer(L, T, opt)) return rc;
  if (T == 0) return TMOE_OK;
  if (!x || !y) return fail(TMOE_ERR_INVALID, "tmoe_moe_forward: null x or y");
  const size_t need = tmoe_moe_workspace_size(L, T, opt);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_moe_forward: workspace %zu < %zu bytes", ws_bytes, need);
  if (T == 0) return TMOE_OK;
  const int H = L->hidden, E = L->num_experts, k = L->top_k, I = L->moe_inter,
            Is = L->shared_inter;
  const int R = T * k, U = R < E ? R : E, G = H / 64;
  const bool prefill = T >= opt_min_tokens(opt);
  const int maxt = max_tiles(R, E);
  Carve c(ws);
  BlockWs b;
  carve_block(c, L, T, opt, &b);
  int32_t* idx = idx_out ? idx_out : b.idx;
  uint16_t* scores = scores_out ? scores_out : b.scores;
  cudaStream_t s = S(stream);

  const uint16_t* wg = Is > 0 ? L->shared_gate_w : nullptr;
  const bool fused_route = !prefill && T <= kDecodeRouteMaxT;
  if (!fused_route)
    TMOE_TRY(launch_router_logits(x, L->router_w, wg, T, H, E, b.logits, b.gate_logit, s),
             "router_logits");
  RoutePlan p{};
  p.order = b.order;
  p.inv = b.inv;
  p.offsets = b.offsets;

  if (!prefill && opt_layer(opt)) {
    const int ns = decode_layer_stages(T, H, E, k, I, Is, decode_layer_ctas());
    if (ns > 0) {
      // the whole layer in one launch
      LayerArgs a{};
      a.x = x;
      a.wr = L->router_w;
      a.wg = wg;
      a.guw = L->gate_up_w;
      a.gus = L->gate_up_s;
      a.gub = L->gate_up_b;
      a.dnw = L->down_w;
      a.dns = L->down_s;
      a.dnb = L->down_b;
      if (Is > 0) {
        a.sguw = L->shared_gate_up_w;
        a.sgus = L->shared_gate_up_s;
        a.sgub = L->shared_gate_up_b;
        a.sdnw = L->shared_down_w;
        a.sdns = L->shared_down_s;
        a.sdnb = L->shared_down_b;
      }
      a.epoch = b.epoch;
      a.gucnt = b.gucnt;
      a.tlog = b.tlog;
      a.tgate = b.tgate;
      a.tseen = b.tseen;
      a.th = b.th;
      a.ths = b.ths;
      a.idx = idx;
      a.scores = scores;
      a.y = y;
      a.T = T;
      a.H = H;
      a.E = E;
      a.k = k;
      a.I = I;
      a.Is = Is;
      TMOE_TRY(launch_decode_layer(a, ns, s), "decode_layer");
      return TMOE_OK;
    }
  }
  if (!prefill) {
    p.uexp = b.uexp;
    p.ustart = b.ustart;
    p.nuniq = b.nuniq;
    if (fused_route) {
      // logits, top-k and plan in one launch; combine counters zeroed
      TMOE_TRY(launch_decode_route(x, L->router_w, wg, T, H, E, k, b.logits, b.gate_logit, idx,
                                   scores, p, b.counters, H / 32, s),
               "decode_route");
    } else {
      TMOE_TRY(launch_router_topk(b.logits, T, E, k, idx, scores, nullptr, s), "router_topk");
      TMOE_TRY(launch_route_plan(idx, R, E, kTileM, 1, p, b.route_scratch, s), "route_plan");
      TMOE_TRY(launch_zero_i32(b.counters + 1, H / 32, s), "zero_counters");
    }
    StreamParams q{};
    q.x = x;
    q.tokens = T == 1 ? 1 : 0;
    q.K = H;
    q.K_sh = H;
    q.W = L->gate_up_w;
    q.S = L->gate_up_s;
    q.B = L->gate_up_b;
    q.N = 2 * I;
    if (Is > 0) {
      q.Wsh = L->shared_gate_up_w;
      q.Ssh = L->shared_gate_up_s;
      q.Bsh = L->shared_gate_up_b;
      q.Nsh = 2 * Is;
      q.out_sh = b.hs;
    }
    q.uexp = b.uexp;
    q.ustart = b.ustart;
    q.nuniq = b.nuniq;
    q.order = b.order;
    q.umax = U;
    q.col_div = k;
    q.nsh = T;
    q.out = b.h;
    TMOE_TRY(launch_gemv_stream(0, q, T, s), "gemv_gate_up");
    StreamParams d{};
    d.h = b.h;
    d.h_sh = b.hs;
    d.K = I;
    d.K_sh = Is;
    d.W = L->down_w;
    d.S = L->down_s;
    d.B = L->down_b;
    d.N = H;
    if (Is > 0) {
      d.Wsh = L->shared_down_w;
      d.Ssh = L->shared_down_s;
      d.Bsh = L->shared_down_b;
      d.Nsh = H;
      d.out_sh = b.part_sh;
      d.gate_logit = b.gate_logit;
    }
    d.uexp = b.uexp;
    d.ustart = b.ustart;
    d.nuniq = b.nuniq;
    d.order = b.order;
    d.umax = U;
    d.col_div = 1;
    d.nsh = T;
    d.out = b.part;
    d.counters = b.counters + 1;
    d.plan_ready = 1;          // the gate_up kernel releases this one after the routing
    d.scores = scores;
    d.T = T;
    d.k = k;
    d.y = y;
    TMOE_TRY(launch_gemv_stream(1, d, T, s), "gemv_down");
    return TMOE_OK;
  }
  TMOE_TRY(launch_router_topk(b.logits, T, E, k, idx, scores, nullptr, s), "router_topk");

  // ---- prefill: expert-sorted grouped GEMMs (int8 or stock bf16 gate_up)
  p.tile_row = b.tile_row;
  p.tile_exp = b.tile_exp;
  p.ntiles = b.ntiles;
  const bool fr = fast_routed(L, opt), fs = fast_shared(L);
  const int rtile = fr ? kSwTileN : kTileM, rmaxt = tiles_for(R, E, rtile);
  TMOE_TRY(launch_route_plan(idx, R, E, rtile, rmaxt, p, b.route_scratch, s), "route_plan");
  const bool i8 = opt_int8(opt);
  const bool d8 = i8 && opt_down_int8(opt);
  const bool tc = tc05_layer(L, opt);
  const int gs = tc ? tc05_srow(G) : G, gi = tc ? tc05_srow(I / 64) : I / 64;
  auto gemm = [&](bool int8, int epi, const GemmParams& P, int ntiles_max) {
    return tc ? launch_gemm_tc05(int8, epi, P, ntiles_max, s)
              : launch_gemm_grouped(int8, epi, P, ntiles_max, s);
  };
  if ((!fr && !i8 && !tc) || (Is > 0 && !fs)) {   // fp16 copy of x (token order)
    if (tc)
      TMOE_TRY(launch_prep_a16_rows(x, T, H, false, nullptr, nullptr, 1, gs, b.sx16p, nullptr,
                                    b.sxsum, s),
               "prep_x");
    else
      TMOE_TRY(launch_prep_x(x, T, H, b.sx16p, b.sxsum, G, 1, s), "prep_x");
  }
  if (fr) {
    const FastRoute rt{b.tile_row, b.tile_exp, b.ntiles, b.offsets, rmaxt, b.order, k, nullptr};
    if (int rc = run_fast(routed_proj(L), x, T, R, i8, d8, rt, b.fr, b.ys, b.order, nullptr, s,
                          kRoutedNames))
      return rc;
  } else {
    GemmParams g{};
    if (tc) {
      // the expert-sorted operand rows: int8 codes (or x) of token order[r] / k
      TMOE_TRY(launch_prep_a16_rows(x, R, H, i8, b.order, nullptr, k, gs,
                                    reinterpret_cast<uint16_t*>(b.xq), i8 ? b.xsc : nullptr, b.xrs,
                                    s),
               i8 ? "quantize_rows" : "prep_x");
      g.A = b.xq;
      g.asc = i8 ? b.xsc : nullptr;
      g.ars = b.xrs;
      g.s_r = gs;
      g.a_nrows = R;
      g.h_srow = gi;
    } else {
      if (i8) TMOE_TRY(launch_quantize_rows(x, T, H, b.xq, b.xsc, b.xrs, s), "quantize_rows");
      g.A = i8 ? static_cast<const void*>(b.xq) : static_cast<const void*>(b.sx16p);
      g.asc = b.xsc;
      g.ars = i8 ? b.xrs : b.sxsum;
      g.s_r = G;
      g.a_rows = b.order;
      g.a_div = k;
    }
    g.s_g = 1;
    g.W = L->gate_up_w;
    g.E = E;
    g.st = L->gate_up_st;
    g.bt = L->gate_up_bt;
    g.tile_row = b.tile_row;
    g.tile_exp = b.tile_exp;
    g.ntiles = b.ntiles;
    g.offsets = b.offsets;
    g.K = H;
    g.N = 2 * I;
    g.hq = b.hq;
    g.hsc = b.hsc;
    g.hrs = b.hrs;
    g.Rpad_h = R;
    g.h16p = b.h16p;
    TMOE_TRY(gemm(i8, d8 ? kEpiSwigluQ8 : kEpiSwigluH16, g, rmaxt), "gemm_gate_up");
    GemmParams dn{};
    dn.A = (d8 && !tc) ? static_cast<const void*>(b.hq) : static_cast<const void*>(b.h16p);
    dn.asc = b.hsc;
    dn.ars = b.hrs;
    dn.s_r = tc ? gi : 1;      // tcgen05: row-major h scalars; mma.sync: [group][row]
    dn.s_g = tc ? 1 : R;
    dn.a_nrows = R;
    dn.W = L->down_w;
    dn.E = E;
    dn.st = L->down_st;
    dn.bt = L->down_bt;
    dn.tile_row = b.tile_row;
    dn.tile_exp = b.tile_exp;
    dn.ntiles = b.ntiles;
    dn.offsets = b.offsets;
    dn.K = I;
    dn.N = H;
    dn.Y = b.ys;
    dn.y_rows = b.order;   // pair-major: the weighted sum reads a token's k rows contiguously
    TMOE_TRY(gemm(d8, kEpiStore, dn, rmaxt), "gemm_down");
  }
  if (Is > 0) {
    const int stile = fs ? kSwTileN : kTileM, st = (T + stile - 1) / stile;
    TMOE_TRY(launch_dense_tiles(T, stile, b.s_tile_row, b.s_tile_exp, b.s_ntiles, b.s_offsets, s),
             "dense_tiles");
    if (fs) {
      const FastRoute rs{b.s_tile_row, b.s_tile_exp, b.s_ntiles, b.s_offsets, st, nullptr, 1,
                         nullptr};
      if (int rc = run_fast(shared_proj(L), x, T, T, false, false, rs, b.fs, b.ys_sh, nullptr,
                            nullptr, s, kSharedNames))
        return rc;
    } else {
      GemmParams sg{};
      const int gsh = tc ? tc05_srow(Is / 64) : Is / 64;
      sg.A = b.sx16p;
      sg.ars = b.sxsum;
      sg.s_r = gs;
      sg.s_g = 1;
      sg.a_nrows = T;
      sg.W = L->shared_gate_up_w;
      sg.E = 1;
      sg.st = L->shared_gate_up_st;
      sg.bt = L->shared_gate_up_bt;
      sg.tile_row = b.s_tile_row;
      sg.tile_exp = b.s_tile_exp;
      sg.ntiles = b.s_ntiles;
      sg.offsets = b.s_offsets;
      sg.K = H;
      sg.N = 2 * Is;
      sg.hrs = b.shrs;
      sg.Rpad_h = T;
      sg.h_srow = gsh;
      sg.h16p = b.sh16p;
      TMOE_TRY(gemm(false, kEpiSwigluH16, sg, st), "gemm_shared_gate_up");
      GemmParams sd{};
      sd.A = b.sh16p;
      sd.ars = b.shrs;
      sd.s_r = tc ? gsh : 1;
      sd.s_g = tc ? 1 : T;
      sd.a_nrows = T;
      sd.W = L->shared_down_w;
      sd.E = 1;
      sd.st = L->shared_down_st;
      sd.bt = L->shared_down_bt;
      sd.tile_row = b.s_tile_row;
      sd.tile_exp = b.s_tile_exp;
      sd.ntiles = b.s_ntiles;
      sd.offsets = b.s_offsets;
      sd.K = Is;
      sd.N = H;
      sd.Y = b.ys_sh;
      TMOE_TRY(gemm(false, kEpiStore, sd, st), "gemm_shared_down");
    }
  }
  TMOE_TRY(launch_wsum(b.ys, nullptr, scores, T, k, H, opt_wsum(opt), Is > 0 ? b.ys_sh : nullptr,
                       b.gate_logit, y, s),
           "weighted_sum");
  return TMOE_OK;
}

// ------------------------------------------------------- decoder sub-layer

int tmoe_rmsnorm(const uint16_t* x, const uint16_t* weight, int T, int H, float eps, uint16_t* out,
                 void* stream) {
  if (!x || !weight || !out || T < 0 || H <= 0 || !(eps >= 0.0f))
    return fail(TMOE_ERR_INVALID, "tmoe_rmsnorm: bad arguments");
  TMOE_TRY(launch_rmsnorm(x, weight, T, H, eps, out, S(stream)), "rmsnorm");
  return TMOE_OK;
}

int tmoe_residual_inject(const uint16_t* branch, const uint16_t* residual, const uint16_t* weights,
                         int T, int H, int nstreams, uint16_t* out, void* stream) {
  if (!branch || !residual || !out || T < 0 || H <= 0 || nstreams < 0 || nstreams > 64 ||
      (nstreams > 0 && !weights))
    return fail(TMOE_ERR_INVALID, "tmoe_residual_inject: bad arguments");
  TMOE_TRY(launch_inject(branch, residual, weights, T, H, nstreams, out, S(stream)), "inject");
  return TMOE_OK;
}

size_t tmoe_moe_sublayer_workspace_size(const tmoe_layer* L, int T, const tmoe_options* opt) {
  if (!L || T < 0) return 0;
  Carve c(nullptr);
  c.take<uint16_t>((size_t)T * L->hidden);     // normed x
  c.take<uint16_t>((size_t)T * L->hidden);     // the block's output
  c.off = (c.off + 255) & ~size_t(255);
  return c.off + tmoe_moe_workspace_size(L, T, opt);
}

int tmoe_moe_sublayer(const tmoe_layer* L, const uint16_t* norm_weight, float eps,
                      const uint16_t* h, int T, const uint16_t* residual,
                      const uint16_t* inject_weights, int nstreams, const tmoe_options* opt,
                      void* ws, size_t ws_bytes, uint16_t* out, void* stream) {
  if (!L || !norm_weight || T < 0 || nstreams < 0 || nstreams > 64 ||
      (T > 0 && (!h || !out || (nstreams > 0 && (!residual || !inject_weights)))))
    return fail(TMOE_ERR_INVALID, "tmoe_moe_sublayer: bad arguments");
  if (int rc = check_layer(L, T, opt)) return rc;
  if (T == 0) return TMOE_OK;
  const size_t need = tmoe_moe_sublayer_workspace_size(L, T, opt);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_moe_sublayer: workspace %zu < %zu bytes", ws_bytes, need);
  const int H = L->hidden;
  Carve c(ws);
  uint16_t* xn = c.take<uint16_t>((size_t)T * H);
  uint16_t* y = c.take<uint16_t>((size_t)T * H);
  c.off = (c.off + 255) & ~size_t(255);
  void* bws = static_cast<uint8_t*>(ws) + c.off;
  cudaStream_t s = S(stream);
  TMOE_TRY(launch_rmsnorm(h, norm_weight, T, H, eps, xn, s), "rmsnorm");
  if (int rc = tmoe_moe_forward(L, xn, T, opt, bws, ws_bytes - c.off, y, nullptr, nullptr, stream))
    return rc;
  TMOE_TRY(launch_inject(y, nstreams > 0 ? residual : h, inject_weights, T, H, nstreams, out, s),
           "inject");
  return TMOE_OK;
}

}  // extern "C"

// ------------------------------------------------- routed experts on pairs
// The owner side of expert parallelism: rows x [R, H] received from other
// ranks and the (row, local expert) pairs this rank serves.  Same grouped
// GEMMs as the prefill path; y_pairs [P, H] gets each pair's bf16 expert
// output in pair order, exactly the values the single-device block weighs.

namespace {

struct ExpertsWs {
  int32_t *order, *inv, *offsets, *tile_row, *tile_exp, *ntiles;
  void* route_scratch;
  int8_t *xq, *hq;
  float *xsc, *xrs, *hsc, *hrs;
  uint16_t *x16p, *h16p;
  float* xsum;
  FastWs fr;
};

size_t carve_experts(Carve& c, const tmoe_layer* L, int R, int P, const tmoe_options* opt,
                     ExpertsWs* out) {
  const int H = L->hidden, E = L->num_experts, I = L->moe_inter, G = H / 64;
  const int maxt = max_tiles(P, E);
  const bool i8 = opt_int8(opt), d8 = i8 && opt_down_int8(opt), tc = tc05_layer(L, opt);
  const int gs = tc ? tc05_srow(G) : G, gi = tc ? tc05_srow(I / 64) : I / 64;
  ExpertsWs b{};
  b.order = c.take<int32_t>(P);
  b.inv = c.take<int32_t>(P);
  b.offsets = c.take<int32_t>(E + 1);
  b.tile_row = c.take<int32_t>(maxt);
  b.tile_exp = c.take<int32_t>(maxt);
  b.ntiles = c.take<int32_t>(1);
  b.route_scratch = c.take<uint8_t>(route_plan_scratch_bytes(P, E));
  if (fast_routed(L, opt)) {
    carve_fast(c, R, P, H, I, &b.fr);
    if (out) *out = b;
    return c.off;
  }
  if (tc) {  // expert-sorted fp16 rows, one per pair (int8 codes or x) + row scalars
    b.xq = c.take<int8_t>((size_t)P * H * 2);
    b.xsc = c.take<float>((size_t)P * gs);
    b.xrs = c.take<float>((size_t)P * gs);
  } else if (i8) {
    b.xq = c.take<int8_t>((size_t)R * H);
    b.xsc = c.take<float>((size_t)R * G);
    b.xrs = c.take<float>((size_t)R * G);
  } else {
    b.x16p = c.take<uint16_t>((size_t)R * H);
    b.xsum = c.take<float>((size_t)R * G);
  }
  if (d8 && !tc)
    b.hq = c.take<int8_t>((size_t)P * I);
  else
    b.h16p = c.take<uint16_t>((size_t)P * I);
  if (d8) b.hsc = c.take<float>((size_t)P * gi);
  b.hrs = c.take<float>((size_t)P * gi);
  if (out) *out = b;
  return c.off;
}

}  // namespace

extern "C" {

size_t tmoe_moe_experts_workspace_size(const tmoe_layer* L, int R, int npairs,
                                       const tmoe_options* opt) {
  if (!L || R < 0 || npairs < 0) return 0;
  Carve c(nullptr);
  return carve_experts(c, L, R, npairs, opt, nullptr);
}

}  // extern "C"

namespace {
// The owner side; the output row of pair p goes to y_pairs[p] or, when
// y_ptr is set, to y_ptr[p].  With slot_k > 0 there is no pair_row: pair p
// reads row p / slot_k, and pairs whose expert id is negative are skipped.
int moe_experts(const tmoe_layer* L, const uint16_t* x, int R, const int32_t* pair_row,
                int slot_k, const int32_t* pair_exp, int npairs, const tmoe_options* opt,
                void* ws, size_t ws_bytes, uint16_t* y_pairs, uint16_t* const* y_ptr,
                void* stream) {
  if (!L || R < 0 || npairs < 0) return fail(TMOE_ERR_INVALID, "tmoe_moe_experts: bad arguments");
  const int H = L->hidden, E = L->num_experts, I = L->moe_inter, G = H / 64;
  if (!L->gate_up_w || !L->gate_up_st || !L->gate_up_bt || !L->down_w || !L->down_st ||
      !L->down_bt)
    return fail(TMOE_ERR_INVALID, "tmoe_moe_experts: missing routed weights or prepared tables");
  if (H <= 0 || H % 128 || I <= 0 || I % 64 || E <= 0 || E > 1024)
    return fail(TMOE_ERR_UNSUPPORTED, "tmoe_moe_experts: need H %% 128 == 0, I %% 64 == 0, E <= 1024");
  if (R == 0 || npairs == 0) return TMOE_OK;
  if (!x || (!y_pairs && !y_ptr) || (!pair_row && slot_k <= 0) || !pair_exp)
    return fail(TMOE_ERR_INVALID, "tmoe_moe_experts: null pointer");
  const size_t need = tmoe_moe_experts_workspace_size(L, R, npairs, opt);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_moe_experts: workspace %zu < %zu bytes", ws_bytes, need);
  cudaStream_t s = S(stream);
  Carve c(ws);
  ExpertsWs b;
  carve_experts(c, L, R, npairs, opt, &b);
  const int P = npairs;
  const bool fastr = fast_routed(L, opt);
  const int maxt = tiles_for(P, E, fastr ? kSwTileN : kTileM);
  RoutePlan p{};
  p.order = b.order;
  p.inv = b.inv;
  p.offsets = b.offsets;
  p.tile_row = b.tile_row;
  p.tile_exp = b.tile_exp;
  p.ntiles = b.ntiles;
  TMOE_TRY(launch_route_plan(pair_exp, P, E, fastr ? kSwTileN : kTileM, maxt, p, b.route_scratch,
                             s),
           "route_plan");
  const bool i8 = opt_int8(opt), d8 = i8 && opt_down_int8(opt), tc = tc05_layer(L, opt);
  const int gs = tc ? tc05_srow(G) : G, gi = tc ? tc05_srow(I / 64) : I / 64;
  if (fastr) {
    const FastRoute rt{b.tile_row, b.tile_exp, b.ntiles, b.offsets, maxt, b.order,
                       slot_k > 0 ? slot_k : 1, slot_k > 0 ? nullptr : pair_row};
    return run_fast(routed_proj(L), x, R, P, i8, d8, rt, b.fr, y_pairs, b.order, y_ptr, s,
                    kRoutedNames);
  }
  auto gemm = [&](bool int8, int epi, const GemmParams& Pm) {
    return tc ? launch_gemm_tc05(int8, epi, Pm, maxt, s) : launch_gemm_grouped(int8, epi, Pm, maxt, s);
  };
  GemmParams g{};
  if (tc) {
    // one expert-sorted operand row per pair: sorted position -> pair -> row
    TMOE_TRY(launch_prep_a16_rows(x, P, H, i8, b.order, slot_k > 0 ? nullptr : pair_row,
                                  slot_k > 0 ? slot_k : 1, gs, reinterpret_cast<uint16_t*>(b.xq),
                                  i8 ? b.xsc : nullptr, b.xrs, s),
             i8 ? "quantize_rows" : "prep_x");
    g.A = b.xq;
    g.asc = i8 ? b.xsc : nullptr;
    g.ars = b.xrs;
    g.s_r = gs;
    g.a_nrows = P;
    g.h_srow = gi;
  } else {
    if (i8)
      TMOE_TRY(launch_quantize_rows(x, R, H, b.xq, b.xsc, b.xrs, s), "quantize_rows");
    else
      TMOE_TRY(launch_prep_x(x, R, H, b.x16p, b.xsum, G, 1, s), "prep_x");
    g.A = i8 ? static_cast<const void*>(b.xq) : static_cast<const void*>(b.x16p);
    g.asc = b.xsc;
    g.ars = i8 ? b.xrs : b.xsum;
    g.s_r = G;
    g.a_rows = b.order;          // sorted position -> pair
    g.a_map = slot_k > 0 ? nullptr : pair_row;   // pair -> received row
    g.a_div = slot_k > 0 ? slot_k : 1;
  }
  g.s_g = 1;
  g.W = L->gate_up_w;
  g.E = E;
  g.st = L->gate_up_st;
  g.bt = L->gate_up_bt;
  g.tile_row = b.tile_row;
  g.tile_exp = b.tile_exp;
  g.ntiles = b.ntiles;
  g.offsets = b.offsets;
  g.K = H;
  g.N = 2 * I;
  g.hq = b.hq;
  g.hsc = b.hsc;
  g.hrs = b.hrs;
  g.Rpad_h = P;
  g.h16p = b.h16p;
  TMOE_TRY(gemm(i8, d8 ? kEpiSwigluQ8 : kEpiSwigluH16, g), "gemm_gate_up");
  GemmParams dn{};
  dn.A = (d8 && !tc) ? static_cast<const void*>(b.hq) : static_cast<const void*>(b.h16p);
  dn.asc = b.hsc;
  dn.ars = b.hrs;
  dn.s_r = tc ? gi : 1;      // tcgen05: row-major h scalars; mma.sync: [group][row]
  dn.s_g = tc ? 1 : P;
  dn.a_nrows = P;
  dn.W = L->down_w;
  dn.E = E;
  dn.st = L->down_st;
  dn.bt = L->down_bt;
  dn.tile_row = b.tile_row;
  dn.tile_exp = b.tile_exp;
  dn.ntiles = b.ntiles;
  dn.offsets = b.offsets;
  dn.K = I;
  dn.N = H;
  dn.Y = y_pairs;
  dn.y_rows = b.order;         // stored back in pair order
  dn.y_ptr = y_ptr;
  TMOE_TRY(gemm(d8, kEpiStore, dn), "gemm_down");
  return TMOE_OK;
}
}  // namespace

extern "C" {

int tmoe_moe_experts(const tmoe_layer* L, const uint16_t* x, int R, const int32_t* pair_row,
                     const int32_t* pair_exp, int npairs, const tmoe_options* opt, void* ws,
                     size_t ws_bytes, uint16_t* y_pairs, void* stream) {
  return moe_experts(L, x, R, pair_row, 0, pair_exp, npairs, opt, ws, ws_bytes, y_pairs,
                     nullptr, stream);
}

int tmoe_moe_experts_slots(const tmoe_layer* L, const uint16_t* x, int R, const int32_t* slot_exp,
                           const tmoe_options* opt, void* ws, size_t ws_bytes,
                           uint16_t* const* y_rows, void* stream) {
  if (!L || R < 0) return fail(TMOE_ERR_INVALID, "tmoe_moe_experts_slots: bad arguments");
  if (R > 0 && (!y_rows || !slot_exp))
    return fail(TMOE_ERR_INVALID, "tmoe_moe_experts_slots: null pointer");
  const int k = L->top_k;
  if (k <= 0 || (long long)R * k > (1ll << 30))
    return fail(TMOE_ERR_INVALID, "tmoe_moe_experts_slots: bad top_k or too many slots");
  return moe_experts(L, x, R, nullptr, k, slot_exp, R * k, opt, ws, ws_bytes, nullptr, y_rows,
                     stream);
}

// The source side: the block's weighted sum (clone or fast mode) over every
// token's k expert outputs, wherever they were computed, plus the gated
// shared expert — the last step of tmoe_moe_forward.
// ------------------------------------------------ the token-local part of a layer

namespace {
tmoe_options local_options(const tmoe_options* opt) {
  tmoe_options o = opt ? *opt : tmoe_options{512, 1, 0, 1, 0, 0};
  o.min_tokens = 1;   // the prefill (grouped-GEMM) semantics at every T
  return o;
}
}  // namespace

size_t tmoe_moe_local_workspace_size(const tmoe_layer* L, int T, const tmoe_options* opt) {
  if (!L || T < 0) return 0;
  const tmoe_options o = local_options(opt);
  Carve c(nullptr);
  return carve_block(c, L, T, &o, nullptr);
}

int tmoe_moe_local(const tmoe_layer* L, const uint16_t* x, int T, const tmoe_options* opt,
                   void* ws, size_t ws_bytes, int32_t* idx, uint16_t* scores, float* gate_logit,
                   uint16_t* shared_out, void* stream) {
  if (!L) return fail(TMOE_ERR_INVALID, "tmoe_moe_local: null layer");
  const int H = L->hidden, E = L->num_experts, k = L->top_k, Is = L->shared_inter;
  if (T < 0 || Is < 0) return fail(TMOE_ERR_INVALID, "tmoe_moe_local: bad sizes");
  if (int rc = check_router(T, H, E, k)) return rc;
  if (!L->router_w) return fail(TMOE_ERR_INVALID, "tmoe_moe_local: missing router weight");
  if (Is > 0) {
    if (!L->shared_gate_up_w || !L->shared_gate_up_st || !L->shared_gate_up_bt ||
        !L->shared_down_w || !L->shared_down_st || !L->shared_down_bt || !L->shared_gate_w)
      return fail(TMOE_ERR_INVALID, "tmoe_moe_local: the shared expert needs weights and tables");
    if (Is % 64) return fail(TMOE_ERR_UNSUPPORTED, "tmoe_moe_local: need Is %% 64 == 0");
    if (!shared_out || !gate_logit)
      return fail(TMOE_ERR_INVALID, "tmoe_moe_local: null shared_out or gate_logit");
  }
  if (T == 0) return TMOE_OK;
  if (!x || !idx || !scores) return fail(TMOE_ERR_INVALID, "tmoe_moe_local: null x, idx or scores");
  const tmoe_options o = local_options(opt);
  const size_t need = tmoe_moe_local_workspace_size(L, T, opt);
  if (!ws || ws_bytes < need)
    return fail(TMOE_ERR_WORKSPACE, "tmoe_moe_local: workspace %zu < %zu bytes", ws_bytes, need);
  const int G = H / 64;
  Carve c(ws);
  BlockWs b;
  carve_block(c, L, T, &o, &b);
  cudaStream_t s = S(stream);
  const uint16_t* wg = Is > 0 ? L->shared_gate_w : nullptr;
  // the block's prefill steps, the same kernels and arguments
  TMOE_TRY(launch_router_logits(x, L->router_w, wg, T, H, E, b.logits,
                                Is > 0 ? gate_logit : b.gate_logit, s),
           "router_logits");
  TMOE_TRY(launch_router_topk(b.logits, T, E, k, idx, scores, nullptr, s), "router_topk");
  if (Is == 0) return TMOE_OK;
  if (fast_shared(L)) {
    const int st = (T + kSwTileN - 1) / kSwTileN;
    TMOE_TRY(launch_dense_tiles(T, kSwTileN, b.s_tile_row, b.s_tile_exp, b.s_ntiles, b.s_offsets,
                                s),
             "dense_tiles");
    const FastRoute rs{b.s_tile_row, b.s_tile_exp, b.s_ntiles, b.s_offsets, st, nullptr, 1, nullptr};
    return run_fast(shared_proj(L), x, T, T, false, false, rs, b.fs, shared_out, nullptr, nullptr,
                    s, kSharedNames);
  }
  const bool tc = tc05_layer(L, &o);
  const int gs = tc ? tc05_srow(G) : G, gsh = tc ? tc05_srow(Is / 64) : Is / 64;
  if (tc)
    TMOE_TRY(launch_prep_a16_rows(x, T, H, false, nullptr, nullptr, 1, gs, b.sx16p, nullptr,
                                  b.sxsum, s),
             "prep_x");
  else
    TMOE_TRY(launch_prep_x(x, T, H, b.sx16p, b.sxsum, G, 1, s), "prep_x");
  auto gemm = [&](int epi, const GemmParams& P, int ntiles_max) {
    return tc ? launch_gemm_tc05(false, epi, P, ntiles_max, s)
              : launch_gemm_grouped(false, epi, P, ntiles_max, s);
  };
  const int st = (T + kTileM - 1) / kTileM;
  TMOE_TRY(launch_dense_tiles(T, kTileM, b.s_tile_row, b.s_tile_exp, b.s_ntiles, b.s_offsets, s),
           "dense_tiles");
  GemmParams sg{};
  sg.A = b.sx16p;
  sg.ars = b.sxsum;
  sg.s_r = gs;
  sg.s_g = 1;
  sg.a_nrows = T;
  sg.W = L->shared_gate_up_w;
  sg.E = 1;
  sg.st = L->shared_gate_up_st;
  sg.bt = L->shared_gate_up_bt;
  sg.tile_row = b.s_tile_row;
  sg.tile_exp = b.s_tile_exp;
  sg.ntiles = b.s_ntiles;
  sg.offsets = b.s_offsets;
  sg.K = H;
  sg.N = 2 * Is;
  sg.hrs = b.shrs;
  sg.Rpad_h = T;
  sg.h_srow = gsh;
  sg.h16p = b.sh16p;
  TMOE_TRY(gemm(kEpiSwigluH16, sg, st), "gemm_shared_gate_up");
  GemmParams sd{};
  sd.A = b.sh16p;
  sd.ars = b.shrs;
  sd.s_r = tc ? gsh : 1;
  sd.s_g = tc ? 1 : T;
  sd.a_nrows = T;
  sd.W = L->shared_down_w;
  sd.E = 1;
  sd.st = L->shared_down_st;
  sd.bt = L->shared_down_bt;
  sd.tile_row = b.s_tile_row;
  sd.tile_exp = b.s_tile_exp;
  sd.ntiles = b.s_ntiles;
  sd.offsets = b.s_offsets;
  sd.K = Is;
  sd.N = H;
  sd.Y = shared_out;
  TMOE_TRY(gemm(kEpiStore, sd, st), "gemm_shared_down");
  return TMOE_OK;
}

// ------------------------------------------- expert-parallel peer exchanges

size_t tmoe_ep_buffer_bytes(int world, int cap, int H, int k, int T_max, size_t* offsets) {
  size_t off[4];
  if (world <= 0 || cap < 0 || H <= 0 || k <= 0 || T_max < 0) return 0;
  const size_t n = ep_layout(world, cap, H, k, T_max, off);
  if (offsets)
    for (int i = 0; i < 4; ++i) offsets[i] = off[i];
  return n;
}

int tmoe_ep_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(TMOE_ERR_INVALID, "tmoe_ep_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return fail(TMOE_ERR_CUDA, "tmoe_ep_alloc: %s", cudaGetErrorString(e));
  return TMOE_OK;
}

int tmoe_ep_free(void* ptr) {
  if (ptr) {
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) return fail(TMOE_ERR_CUDA, "tmoe_ep_free: %s", cudaGetErrorString(e));
  }
  return TMOE_OK;
}

int tmoe_ipc_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return fail(TMOE_ERR_INVALID, "tmoe_ipc_handle: null argument");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return fail(TMOE_ERR_CUDA, "tmoe_ipc_handle: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  return TMOE_OK;
}

int tmoe_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(TMOE_ERR_INVALID, "tmoe_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(TMOE_ERR_CUDA, "tmoe_ipc_open: %s", cudaGetErrorString(e));
  return TMOE_OK;
}

int tmoe_ipc_close(void* ptr) {
  if (ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return fail(TMOE_ERR_CUDA, "tmoe_ipc_close: %s", cudaGetErrorString(e));
  }
  return TMOE_OK;
}

int tmoe_ep_dispatch(const uint16_t* x, const int32_t* idx, int T, int k, int H,
                     int experts_per_rank, int world, int rank, void* const* peers,
                     const size_t* offsets, int cap, int epoch, int32_t* counters, void* stream) {
  if (T < 0 || k <= 0 || k >= 128 || H <= 0 || H % 8 || experts_per_rank <= 0 || world <= 0 ||
      world > 32 || rank < 0 || rank >= world || T > cap || !peers || !offsets || !counters ||
      (T > 0 && (!x || !idx)))
    return fail(TMOE_ERR_INVALID, "tmoe_ep_dispatch: bad arguments");
  EpDispatchArgs a{};
  a.x = x;
  a.idx = idx;
  a.peer = peers;
  a.off_x = offsets[0];
  a.off_meta = offsets[1];
  a.off_flags = offsets[3];
  a.counters = counters;
  a.T = T;
  a.k = k;
  a.H = H;
  a.epr = experts_per_rank;
  a.world = world;
  a.rank = rank;
  a.cap = cap;
  a.epoch = epoch;
  TMOE_TRY(launch_ep_dispatch(a, S(stream)), "ep_dispatch");
  return TMOE_OK;
}

int tmoe_ep_slots(const void* own, const size_t* offsets, const int32_t* rows_in, int world,
                  int cap, int k, int experts_per_rank, int H, void* const* peers,
                  int32_t* slot_exp, uint16_t** y_rows, void* stream) {
  if (!own || !offsets || !rows_in || world <= 0 || world > 32 || cap < 0 || k <= 0 ||
      experts_per_rank <= 0 || H <= 0 || !peers || !slot_exp || !y_rows)
    return fail(TMOE_ERR_INVALID, "tmoe_ep_slots: bad arguments");
  EpSlotsArgs a{};
  a.meta = reinterpret_cast<const int32_t*>(static_cast<const uint8_t*>(own) + offsets[1]);
  a.rows_in = rows_in;
  a.peer = peers;
  a.off_ret = offsets[2];
  a.slot_exp = slot_exp;
  a.y_rows = reinterpret_cast<unsigned long long*>(y_rows);
  a.world = world;
  a.cap = cap;
  a.k = k;
  a.epr = experts_per_rank;
  a.H = H;
  TMOE_TRY(launch_ep_slots(a, S(stream)), "ep_slots");
  return TMOE_OK;
}

int tmoe_ep_wait(const void* own, const size_t* offsets, int which, int world, int epoch,
                 int32_t* counts, void* stream) {
  if (!own || !offsets || (which != 0 && which != 1) || world <= 0 || world > 32 || !counts)
    return fail(TMOE_ERR_INVALID, "tmoe_ep_wait: bad arguments");
  const unsigned long long* flags = reinterpret_cast<const unsigned long long*>(
      static_cast<const uint8_t*>(own) + offsets[3]) + (size_t)which * world;
  TMOE_TRY(launch_ep_wait(flags, world, epoch, counts, S(stream)), "ep_wait");
  return TMOE_OK;
}

int tmoe_ep_post(int which, const int32_t* counts, int world, int rank, void* const* peers,
                 const size_t* offsets, int epoch, void* stream) {
  if ((which != 0 && which != 1) || world <= 0 || world > 32 || rank < 0 || rank >= world ||
      !peers || !offsets)
    return fail(TMOE_ERR_INVALID, "tmoe_ep_post: bad arguments");
  EpPostArgs a{};
  a.counts = counts;
  a.peer = peers;
  a.off_flags = offsets[3];
  a.which = which;
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  TMOE_TRY(launch_ep_post(a, S(stream)), "ep_post");
  return TMOE_OK;
}

int tmoe_ep_post_return(const int32_t* rows_in, int world, int rank, void* const* peers,
                        const size_t* offsets, int epoch, void* stream) {
  if (!rows_in || world <= 0 || world > 32 || rank < 0 || rank >= world || !peers || !offsets)
    return fail(TMOE_ERR_INVALID, "tmoe_ep_post_return: bad arguments");
  EpPostArgs a{};
  a.poison = rows_in;
  a.npoison = world;
  a.peer = peers;
  a.off_flags = offsets[3];
  a.which = 1;
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  TMOE_TRY(launch_ep_post(a, S(stream)), "ep_post");
  return TMOE_OK;
}

int tmoe_ep_guard(const int32_t* counts, int world, uint16_t* y, int64_t n, void* stream) {
  if (!counts || world <= 0 || world > 32 || n < 0 || (n > 0 && !y))
    return fail(TMOE_ERR_INVALID, "tmoe_ep_guard: bad arguments");
  TMOE_TRY(launch_ep_guard(counts, world, y, (long long)n, S(stream)), "ep_guard");
  return TMOE_OK;
}

int tmoe_moe_combine(const uint16_t* ys, const int32_t* inv, const uint16_t* scores, int T, int k,
                     int D, int mode, const uint16_t* shared_out, const float* gate_logit,
                     uint16_t* y, void* stream) {
  if (!ys || !scores || !y || T < 0 || k <= 0 || (mode != 0 && mode != 1) ||
      (!shared_out) != (!gate_logit))
    return fail(TMOE_ERR_INVALID, "tmoe_moe_combine: bad arguments");
  if (D <= 0 || D % 8) return fail(TMOE_ERR_UNSUPPORTED, "tmoe_moe_combine: need D %% 8 == 0");
  TMOE_TRY(launch_wsum(ys, inv, scores, T, k, D, mode, shared_out, gate_logit, y, S(stream)),
           "weighted_sum");
  return TMOE_OK;
}

}  // extern "C"
