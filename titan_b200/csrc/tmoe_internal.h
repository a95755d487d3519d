// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tmoe {

constexpr int kSmallRows = 2048;   // route plans up to this many rows use one CTA
constexpr int kTileM = 128;        // grouped-GEMM row tile
constexpr int kEpiStore = 0;       // bf16 store
constexpr int kEpiSwigluQ8 = 1;    // SwiGLU + int8 requantisation of h
constexpr int kEpiSwigluH16 = 2;   // SwiGLU + fp16 operand copy of h

struct RoutePlan {
  int32_t* order;       // [R] sorted row -> flat (token*k + slot)
  int32_t* inv;         // [R] flat -> sorted row
  int32_t* offsets;     // [E+1]
  int32_t* sorted_ids;  // [R] expert of each sorted row (optional)
  int32_t* tile_row;    // [maxt] (optional)
  int32_t* tile_exp;    // [maxt]
  int32_t* ntiles;      // [1]
  int32_t* uexp;        // [min(R,E)] distinct experts, ascending (optional)
  int32_t* ustart;      // [min(R,E)+1] first sorted row of each distinct expert, then R
  int32_t* nuniq;       // [1]
};

struct GemmParams {
  const void* A;        // I8: int8 codes [rows][K]; F16: fp16 operand layout [rows][K]
  const float* asc;     // row scale (I8 only), element (row, g) at row*s_r + g*s_g
  const float* ars;     // exact group sum of the unquantised row, same strides
  long long s_r, s_g;
  const int32_t* a_rows;  // optional: sorted row r reads A row a_rows[r] / a_div,
  int a_div;              // or a_map[a_rows[r]] when a_map is set
  const int32_t* a_map;
  int E;                // experts in W / st / bt (tcgen05 kernel: TMA map extents)
  const uint32_t* W;    // [E][N][K/8] packed int4
  const uint16_t* st;   // [E][G][N] bf16 scales
  const uint16_t* bt;   // [E][G][N] bf16 biases
  const int32_t* tile_row;
  const int32_t* tile_exp;
  const int32_t* ntiles;
  const int32_t* offsets;  // [E+1]
  int K, N;             // N = weight rows (2I for the SwiGLU epilogues)
  uint16_t* Y;          // store: bf16 [R][N]
  const int32_t* y_rows;  // optional: sorted row r is stored at Y row y_rows[r]
  uint16_t* const* y_ptr;  // optional: Y row i is stored at y_ptr[i] (any device's memory)
  int8_t* hq;           // SwiGLU-Q8: int8 h [Rpad][N/2]
  float* hsc;           // [N/128][Rpad_h]
  float* hrs;           // [N/128][Rpad_h]
  int Rpad_h;
  int h_srow;           // tcgen05 kernel: h scalars are written row-major, [rows][h_srow]
  int a_nrows;          // tcgen05 kernel: rows of A (expert-sorted, contiguous; TMA extent)
  uint16_t* h16p;       // SwiGLU-H16: fp16 operand layout [Rpad][N/2]
  uint16_t* hbf;        // optional bf16 h [R][N/2]
};


// Streaming decode GEMV over the distinct experts (decode.cu).
struct StreamParams {
  const uint16_t* x;      // modes 0/2: bf16 activation rows [rows][K]; the row of sorted
                          // column p is order[p] / col_div (shared expert: column = token)
  const float* h;         // mode 1: routed fp32 h [R][K]
  const float* h_sh;      // mode 1: shared fp32 h [T][K_sh]
  int K, K_sh;
  const uint32_t* W;      // routed weights [E][N][K/8], scales / biases [E][N][K/64]
  const uint16_t* S;
  const uint16_t* B;
  int N;
  const uint32_t* Wsh;    // shared expert [Nsh][K_sh/8] or null
  const uint16_t* Ssh;
  const uint16_t* Bsh;
  int Nsh;
  const int32_t* uexp;
  const int32_t* ustart;
  const int32_t* nuniq;
  const int32_t* order;
  int umax;
  int col_div;
  int nsh;                // shared-expert columns (tokens)
  float* out;             // modes 0/1: routed fp32 output rows order[p]
  float* out_sh;          // modes 0/1: shared fp32 output rows t
  uint16_t* outb;         // mode 2: bf16 output rows order[p]
  int32_t* counters;      // mode 1: [N/32] slab counters, zero on entry, left zero
  const uint16_t* scores; // mode 1: bf16 [T][k] (or scores_f32)
  const float* scores_f32;
  const float* gate_logit;  // mode 1 with a shared expert: fp32 [T]
  int T, k;
  uint16_t* y;            // mode 1: bf16 [T][N]
  int tokens;             // modes 0/2: number of activation rows when known to be 1
                          // (then every column is row 0), else 0
  int plan_ready;         // mode 1: the routing was complete when the previous kernel
                          // released this launch (it reads it before its wait)
};

size_t gemv_stream_smem(int K, int ncol, bool lo);
int gemv_slab_rows();
// max_cols: an upper bound of the columns (activation rows) of any one expert
cudaError_t launch_gemv_stream(int mode, const StreamParams& P, int max_cols, cudaStream_t s);
cudaError_t launch_zero_i32(int32_t* p, int n, cudaStream_t s);
// Router logits + top-k + plan for T <= kDecodeRouteMaxT in one launch.
// counters[0] (a ticket) must be zero on entry and is zero on exit;
// counters[1..ncounters] are zeroed for the decode combine.
cudaError_t launch_decode_route(const uint16_t* x, const uint16_t* wr, const uint16_t* wg, int T,
                                int H, int E, int k, uint16_t* logits, float* gate_logit,
                                int32_t* idx, uint16_t* scores, const RoutePlan& plan,
                                int32_t* counters, int ncounters, cudaStream_t s);
constexpr int kDecodeRouteMaxT = 8;

cudaError_t launch_router_logits(const uint16_t* x, const uint16_t* wr, const uint16_t* wg, int T,
                                 int H, int E, uint16_t* logits, float* gate_logit, cudaStream_t s);
cudaError_t launch_router_topk(const uint16_t* logits, int T, int E, int k, int32_t* idx,
                               uint16_t* scores, uint16_t* probs_out, cudaStream_t s);
size_t route_plan_scratch_bytes(int R, int E);
cudaError_t launch_route_plan(const int32_t* idx, int R, int E, int tile_m, int maxt,
                              const RoutePlan& plan, void* scratch, cudaStream_t s);
cudaError_t launch_quantize_rows(const uint16_t* x, int R, int K, int8_t* xq, float* xsc,
                                 float* xrs, cudaStream_t s);
cudaError_t launch_gemm_grouped(bool int8, int epi, const GemmParams& P, int maxt, cudaStream_t s);
// tcgen05 version: A operands are fp16 [rows][K] with every 8-element chunk
// in (0,4,1,5,2,6,3,7) order (prep_a16); SwiGLU epilogues write h the same way.
// tcgen05 grouped GEMM: A expert-sorted ([a_nrows][K] fp16, no a_rows / a_map),
// row scalars [a_nrows][s_r] (s_g = 1, s_r a multiple of 4), K <= 3072.
bool gemm_tc05_supported(int K, int N);
cudaError_t launch_gemm_tc05(bool int8, int epi, const GemmParams& P, int maxt, cudaStream_t s);
cudaError_t launch_prep_a16(const uint16_t* x, int R, int K, bool quant, uint16_t* a16, float* xsc,
                            float* xrs, cudaStream_t s);
// Gathered variant: output row m reads x row a_map[a_rows[m]] (a_map set) or
// a_rows[m] / a_div (a_rows set, else m); scalars at m * srow + g.
cudaError_t launch_prep_a16_rows(const uint16_t* x, int R, int K, bool quant, const int32_t* a_rows,
                                 const int32_t* a_map, int a_div, int srow, uint16_t* a16,
                                 float* xsc, float* xrs, cudaStream_t s);
// Scalar row stride of the tcgen05 kernel's operands: groups padded to 4
// (one 16-byte TMA box column per 4 groups).
inline int tc05_srow(int G) { return (G + 3) & ~3; }
int tc05_error_flag();

// Persistent swap-AB grouped GEMM (gemm_sw.cu): weight rows on the MMA's M
// side (two 128-row tiles per work item), up to kSwTileN routed rows of one
// expert on N; one exact MMA per 64-wide group and the reference's per-group
// fp32 FMAs in the epilogue.
constexpr int kSwTileN = 64;       // routed rows per work item (route plan tile size)
struct SwParams {
  const uint16_t* B;       // activation operand rows [brows][K] fp16, each 8-element chunk
                           // in (0,4,1,5,2,6,3,7) order: int8 codes, or x * 2^-Et (stock)
  const float* c1;         // [brows][K/64]: the group's activation scale xsc, or 2^Et
  const float* c2;         // [brows][K/64]: exact group sum of the unquantised row
  const int32_t* b_rows;   // optional: sorted row r reads B row b_rows[r] / b_div,
  int b_div;               // or b_map[b_rows[r]] when b_map is set
  const int32_t* b_map;
  const uint32_t* W;       // [E][Nw][K/8] packed int4
  const uint16_t* st;      // [E][G][Nw] bf16 scales (transposed)
  const uint16_t* bt;      // [E][G][Nw] bf16 biases (transposed)
  const float* rscale;     // [E][Nw] 2^Ew: the weight row's scale normaliser
  int E, K, Nw;
  int bias_bf16;           // bias bf16(b + 8s) (int8 algebra) or fp32 b + 8s (stock)
  const int32_t* tile_row;
  const int32_t* tile_exp;
  const int32_t* ntiles;
  const int32_t* offsets;  // [E+1]
  int maxt;
  uint16_t* Y;             // store: bf16 rows of Nw
  const int32_t* y_rows;   // optional: sorted row r is stored at Y row y_rows[r]
  uint16_t* const* y_ptr;  // optional: Y row i is stored at y_ptr[i] (any device's memory)
  uint16_t* H;             // SwiGLU: bf16 h [R][Nw/2] in sorted row order
};
// epi: kEpiStore or kEpiSwigluH16 (bf16 h).  False: the shape is outside this
// kernel (Nw % 256, K % 256 or 64) and the caller uses the per-group kernel.
bool gemm_sw_supported(int epi, int K, int Nw);
cudaError_t launch_gemm_sw(int epi, const SwParams& P, cudaStream_t s);
// Activation operand rows for gemm_sw, one warp per row: quant = the
// reference's per-(row, 64-group) quantiser (codes xu - 128 as fp16, c1 =
// amax/127, c2 = the exact group sum); else x * 2^-Et with one power of two
// per row (amax * 2^-Et in [2^8, 2^9)), c1 = 2^Et, c2 = the group sums.
// rows_limit (optional, device): rows at or past *rows_limit are left alone.
cudaError_t launch_prep_rows(const uint16_t* x, int R, int K, bool quant, uint16_t* out,
                             float* c1, float* c2, const int32_t* rows_limit, cudaStream_t s);
// rscale[e][n] = 2^Ew with max_g 8|s| * 2^Ew in [2^13, 2^14).
cudaError_t launch_row_scale(const uint16_t* scales, const uint16_t* biases, long long rows, int K,
                             float* rscale, cudaStream_t s);
int sw_error_flag();

// Single-launch decode layer (decode_layer.cu), T <= kLayerMaxT tokens.
struct LayerArgs {
  const uint16_t* x;                                   // [T][H] bf16
  const uint16_t* wr;                                  // router [E][H] bf16
  const uint16_t* wg;                                  // shared-expert gate [H] or null
  const uint32_t* guw; const uint16_t* gus; const uint16_t* gub;     // gate_up [E][2I][..]
  const uint32_t* dnw; const uint16_t* dns; const uint16_t* dnb;     // down [E][H][..]
  const uint32_t* sguw; const uint16_t* sgus; const uint16_t* sgub;  // shared gate_up [2Is][..]
  const uint32_t* sdnw; const uint16_t* sdns; const uint16_t* sdnb;  // shared down [H][..]
  // Exchanges between CTAs (no grid barrier): the logits carry the launch
  // epoch in every word (a reader waits until the tags match); h is
  // published by a release-increment of gucnt per gate_up tile.
  int32_t* epoch;                // launch epoch counter, only this kernel writes it
  unsigned long long* gucnt;     // gate_up tiles finished, all launches (only grows)
  unsigned long long* tlog;      // [T][E] bf16 logit | epoch << 32
  unsigned long long* tgate;     // [T] fp32 gate logit | epoch << 32
  int32_t* tseen;                // [kLayerMaxCtas] epoch seen by each CTA at its start
  uint32_t* th;                  // [T*k][I] h as fp16 hi | fp16 lo << 16
  uint32_t* ths;                 // [T][Is] the same for the shared expert
  int32_t* idx;          // [T][k] out
  uint16_t* scores;      // [T][k] out
  uint16_t* y;           // [T][H] out
  int T, H, E, k, I, Is;
};
constexpr int kLayerMaxT = 4;
constexpr int kLayerMaxCtas = 256;   // the grid is one CTA per SM
// Ring stages for the plan (2..4), or 0 when the shape cannot take this path.
int decode_layer_stages(int T, int H, int E, int k, int I, int Is, int nct);
int decode_layer_ctas();
size_t decode_layer_smem(int T, int H, int E, int k, int I, int Is, int nct, int ns);
cudaError_t launch_decode_layer(const LayerArgs& a, int ns, cudaStream_t s);
int layer_error_flag();
int decode_range_flag();

// Expert-parallel exchanges over peer memory (ep_p2p.cu).
struct EpDispatchArgs {
  const uint16_t* x;        // [T][H] bf16
  const int32_t* idx;       // [T][k] global expert ids
  void* const* peer;        // [W] each rank's exchange allocation, mapped here
  size_t off_x, off_meta, off_flags;
  int32_t* counters;        // [1 + W]: ticket, rows taken per rank; zero between launches
  int T, k, H, epr, world, rank, cap, epoch;
};
struct EpSlotsArgs {
  const int32_t* meta;      // this rank's recv_meta [W][cap][k+1]
  const int32_t* rows_in;   // [W] rows posted by each source (-1: its wait gave up)
  void* const* peer;
  size_t off_ret;
  int32_t* slot_exp;               // [W*cap*k]
  unsigned long long* y_rows;      // [W*cap*k]
  int world, cap, k, epr, H;
};
struct EpPostArgs {
  const int32_t* counts;   // [world] or null (count 0)
  const int32_t* poison;   // [npoison] or null: any negative entry posts count -1
  int npoison;
  void* const* peer;
  size_t off_flags;
  int which, world, rank, epoch;
};
cudaError_t launch_ep_dispatch(const EpDispatchArgs& a, cudaStream_t s);
cudaError_t launch_ep_wait(const unsigned long long* flags, int W, int epoch, int32_t* counts,
                           cudaStream_t s);
cudaError_t launch_ep_post(const EpPostArgs& a, cudaStream_t s);
cudaError_t launch_ep_slots(const EpSlotsArgs& a, cudaStream_t s);
cudaError_t launch_ep_guard(const int32_t* counts, int W, uint16_t* y, long long n, cudaStream_t s);
size_t ep_layout(int world, int cap, int H, int k, int T_max, size_t* off);
int ep_error_flag();
cudaError_t launch_to_f16p(const uint16_t* x, long long n, uint16_t* y, cudaStream_t s);
cudaError_t launch_prep_x(const uint16_t* x, int R, int K, uint16_t* x16p, float* xsum,
                          long long sum_sm, long long sum_sg, cudaStream_t s);
cudaError_t launch_wsum(const uint16_t* ys, const int32_t* inv, const uint16_t* scores, int T, int k,
                        int D, int mode, const uint16_t* sh, const float* gate_logit, uint16_t* out,
                        cudaStream_t s);
cudaError_t launch_swiglu(const uint16_t* gu, int R, int I, uint16_t* h, cudaStream_t s);
cudaError_t launch_affine_quantize(const float* w, long long rows, int K, uint32_t* wq,
                                   uint16_t* scales, uint16_t* biases, cudaStream_t s);
cudaError_t launch_prepare_tables(const uint16_t* scales, const uint16_t* biases, int E, int N, int G,
                                  uint16_t* st, uint16_t* bt, cudaStream_t s);
cudaError_t launch_qsum(const uint32_t* w, int E, int N, int K, uint16_t* qsum, cudaStream_t s);
cudaError_t launch_dense_tiles(int R, int tile_m, int32_t* tile_row, int32_t* tile_exp,
                               int32_t* ntiles, int32_t* offsets, cudaStream_t s);

// Raises `func`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (kernel, device); thread-safe (host_util.cu).
cudaError_t ensure_smem_attr(const void* func, int bytes);
// SMs of the current device, cached per device; thread-safe.
int device_sm_count();
// 2D TMA map over a row-major [rows][cols] array of `esize`-byte elements
// (no interleave, L2 256B promotion, no OOB fill); false if it cannot be made.
bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
               unsigned long long cols, unsigned long long rows, unsigned box_cols,
               unsigned box_rows, CUtensorMapSwizzle sw);

// The decoder-layer steps either side of the block (norm.cu).
cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* w, int T, int H, float eps,
                           uint16_t* out, cudaStream_t s);
cudaError_t launch_inject(const uint16_t* branch, const uint16_t* hyper, const uint16_t* wts, int T,
                          int H, int n, uint16_t* out, cudaStream_t s);

// Records `msg` as this thread's tmoe_last_error() text and returns `code`.
int record_error(int code, const char* msg);

}  // namespace tmoe
