/*
 * titan_moe.h — C ABI of the B200-native quantised mixture-of-experts block.
 *
 * Plain pointers and sizes only.  Every pointer argument is a device pointer
 * unless stated otherwise; `stream` is a cudaStream_t (NULL = the legacy
 * default stream).  No entry point allocates memory: callers pass buffers and
 * a workspace sized by the matching *_workspace_size() query.  No entry point
 * synchronises the host; all launch on `stream` and return immediately.
 *
 * Tensor conventions (MLX layout, as in the reference):
 *   bf16 values are uint16_t bit patterns;
 *   packed int4 weights w [E, N, K/8] uint32, element 8j+i of a word in
 *   bits 4i..4i+3 (low nibble first);  scales/biases [E, N, K/64] bf16;
 *   dequantised weight = q * scale + bias, group size 64, 4 bits, affine.
 *   A fused gate_up tensor holds the gate rows [0, I) then the up rows [I, 2I).
 *
 * Return value: TMOE_OK or an error code; tmoe_last_error() describes the
 * last failure on the calling thread.
 */
#ifndef TITAN_MOE_H
#define TITAN_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TMOE_OK = 0,
  TMOE_ERR_INVALID = 1,     /* bad argument or inconsistent shape            */
  TMOE_ERR_UNSUPPORTED = 2, /* shape outside what the kernels implement      */
  TMOE_ERR_CUDA = 3,        /* a CUDA launch or runtime call failed          */
  TMOE_ERR_NCCL = 4,        /* an NCCL call failed (expert parallelism)      */
  TMOE_ERR_TIMEOUT = 5,     /* a bounded device wait gave up                 */
  TMOE_ERR_WORKSPACE = 6    /* workspace missing or smaller than required    */
};

#define TMOE_ABI_VERSION 4

int tmoe_abi_version(void);
const char* tmoe_last_error(void);

/* Profiling hook (no reference counterpart: the reference times whole MLX
 * graphs).  When set, every entry point calls fn(ctx, name) on the calling
 * host thread immediately before each kernel launch, so a caller can record
 * events on the stream between kernels (and one after the call returns) or
 * count launches.  Per calling thread; NULL disables. */
typedef void (*tmoe_stage_fn)(void* ctx, const char* name);
void tmoe_set_stage_hook(tmoe_stage_fn fn, void* ctx);

/* ------------------------------------------------------------ weight prep */

/* MLX mx.quantize(w, group_size=64, bits=4, mode="affine") on the GPU
 * (call sites: titan/adapters/mlx/vendor/mlx_lm/models/switch_layers.py:42,179).
 * w fp32 [rows, K] -> wq uint32 [rows, K/8], scales/biases bf16 [rows, K/64]. */
int tmoe_affine_quantize(const float* w, int64_t rows, int K, uint32_t* wq, uint16_t* scales,
                         uint16_t* biases, void* stream);

/* Transposed [E, K/64, N] scale and bias tables streamed by the grouped GEMMs.
 * Replaces the table builder of titan/kernels/moe_gather_int8.py:227-248
 * (build_tables / Int8Tables) and engine/patches/moe-int8/kernel.py:432-446
 * (prepare_weights); the int8 kernel folds b + 8s itself and needs no qsum. */
int tmoe_prepare_tables(const uint16_t* scales, const uint16_t* biases, int E, int N, int K,
                        uint16_t* scales_t, uint16_t* biases_t, void* stream);

/* Power-of-two row normalisers rs [E, N] fp32 for the swap-AB grouped GEMM:
 * rs = 2^Ew with max over the row's groups of 8|s| times rs in [2^13, 2^14),
 * so every scaled nibble (q - 8) s rs of the row is an exact fp16 (for scales
 * within 2^24 of the row's largest).  Part of the same one-time table build as
 * tmoe_prepare_tables (titan/kernels/moe_gather_int8.py:227-248,
 * engine/patches/moe-int8/kernel.py:432-446); scales / biases [E, N, K/64]. */
int tmoe_prepare_row_scale(const uint16_t* scales, const uint16_t* biases, int E, int N, int K,
                           float* row_scale, void* stream);

/* Nibble sums qsum [E, K/64, N] uint16 — the reference table of
 * titan/kernels/moe_gather_int8.py:189-202 (titan_i8_qsum), for callers that
 * still hold Int8Tables. */
int tmoe_qsum(const uint32_t* w, int E, int N, int K, uint16_t* qsum, void* stream);

/* -------------------------------------------------------------- activations */

/* Per (row, 64-group) uint8 activation quantiser, zero point 128, scale
 * amax/127 — titan/kernels/moe_gather_int8.py:168-182 (quantize_activations).
 * Writes signed codes xq = xu - 128 [R, K] int8, xsc / xrs [R, K/64] fp32
 * (scale and exact group sum of the unquantised row). */
int tmoe_quantize_activations(const uint16_t* x, int R, int K, int8_t* xq, float* xsc, float* xrs,
                              void* stream);

/* ------------------------------------------------------------------ router */

/* Router Linear + softmax(precise) + top-k + renormalisation —
 * titan/adapters/mlx/vendor/mlx_vlm/models/qwen3_5_moe/language.py:65-71 and the
 * fused router of engine/patches/decode-fusion/fused_kernels.py:348-374.
 * x [T, H] bf16, router_w [E, H] bf16; logits_ws [T, E] bf16 scratch (also the
 * router logits on return); idx [T, k] int32 in selection order (descending
 * probability, lowest index first on ties); scores [T, k] bf16; probs_out
 * [T, E] bf16 or NULL.  E <= 1024, k <= 32, H % 64 == 0. */
int tmoe_router_topk(const uint16_t* x, const uint16_t* router_w, int T, int H, int E, int k,
                     uint16_t* logits_ws, int32_t* idx, uint16_t* scores, uint16_t* probs_out,
                     void* stream);

/* ------------------------------------------------------------ routing plan */

/* Stable sort of flat expert ids and the ragged tile table —
 * switch_layers.py:13-25 (_gather_sort / _scatter_unsort) and
 * titan/kernels/moe_gather_ws.py:176-202 (build_tiles, TileTable).
 * order [R]: sorted row -> flat index; inv_order [R]: flat -> sorted row;
 * offsets [E+1]; tile_row / tile_exp [maxt] (tiles of 128 rows, may be NULL);
 * ntiles [1].  maxt >= ceil(R/128) + E.  Negative ids are left out: their
 * inv_order is -1 and offsets[E] counts the others. */
size_t tmoe_route_workspace_size(int R, int E);
int tmoe_route_sort(const int32_t* idx, int R, int E, void* ws, size_t ws_bytes, int32_t* order,
                    int32_t* inv_order, int32_t* offsets, int32_t* tile_row, int32_t* tile_exp,
                    int32_t* ntiles, int maxt, void* stream);

/* ---------------------------------------------------------------- gathers */

/* int8-activation x int4-weight sorted gather: y[r] = x[r] @ dequant(w[rhs[r]])^T
 * with x quantised per (row, 64-group) — the drop-in for
 * mx.gather_qmm(..., sorted_indices=True) installed by
 * engine/patches/moe-int8/patch.py:105-122 (kernel.py:482-501,
 * titan/kernels/moe_gather_int8.py:393-425).
 * x [R, K] bf16, rhs [R] int32 (sorted by expert), scales_t / biases_t from
 * tmoe_prepare_tables; y [R, N] bf16.  N % 128 == 0, K % 64 == 0. */
size_t tmoe_gather_qmm_int8_workspace_size(int R, int E, int N, int K);
int tmoe_gather_qmm_int8(const uint16_t* x, const uint32_t* w, const uint16_t* scales_t,
                         const uint16_t* biases_t, const int32_t* rhs, int R, int E, int N, int K,
                         void* ws, size_t ws_bytes, uint16_t* y, void* stream);

/* tmoe_gather_qmm_int8 without a workspace argument; it allocates nothing.
 * No counterpart in the reference (MLX allocates its own temporaries).
 * For callers that cannot allocate device memory at the call site: a host
 * binding with no device allocator of its own (a ctypes / cgo stub holding
 * only the input and output pointers), or code running while a serving engine
 * has reserved the whole device memory pool.  Scratch is one fixed array of
 * tmoe_static_scratch_bytes() (16 MiB) per device inside this library's
 * device image; a call whose tmoe_gather_qmm_int8_workspace_size() exceeds it
 * returns TMOE_ERR_WORKSPACE before any launch.  The first call on a device
 * looks the array up (this may load the library's device module): make it
 * before any stream capture.  All calls on a device share the array, so calls
 * in flight at the same time on different streams or host threads race:
 * serialise them on one stream. */
size_t tmoe_static_scratch_bytes(void);
int tmoe_gather_qmm_int8_static(const uint16_t* x, const uint32_t* w, const uint16_t* scales_t,
                                const uint16_t* biases_t, const int32_t* rhs, int R, int E, int N,
                                int K, uint16_t* y, void* stream);

/* bf16-activation gather with exact dequantisation and fp32 accumulation —
 * the stock mx.gather_qmm of switch_layers.py:86-98 (sorted or unsorted rhs).
 * x [R, K] bf16, rhs [R] int32 (any order); scales_t / biases_t may be NULL
 * when R <= 256 (decode GEMV path), otherwise required; y [R, N] bf16.
 * N % 128 == 0, K % 64 == 0. */
size_t tmoe_gather_qmm_bf16_workspace_size(int R, int E, int N, int K);
int tmoe_gather_qmm_bf16(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                         const uint16_t* biases, const uint16_t* scales_t,
                         const uint16_t* biases_t, const int32_t* rhs, int R, int E, int N, int K,
                         void* ws, size_t ws_bytes, uint16_t* y, void* stream);

/* ------------------------------------------------------- decode-fused ops */

/* h[t, j, :] = silu(Wg[e] x_t) * (Wu[e] x_t), fp32 —
 * engine/patches/decode-fusion/fused_kernels.py:194-210 (gate_up_silu).
 * x [T, K] bf16, w [E, 2I, K/8], idx [T, k]; h [T, k, I] fp32. */
size_t tmoe_decode_workspace_size(int T, int k, int E, int K, int I);
int tmoe_gate_up_silu(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                      const uint16_t* biases, const int32_t* idx, int T, int k, int E, int K, int I,
                      void* ws, size_t ws_bytes, float* h, void* stream);

/* y[t] = sum_j scores[t, j] * (Wd[idx[t, j]] h[t, j]) in fp32, bf16 out —
 * fused_kernels.py:213-229 (down_wsum).  h [T, k, I] fp32, w [E, D, I/8],
 * scores [T, k] fp32; y [T, D] bf16. */
int tmoe_down_wsum(const float* h, const uint32_t* w, const uint16_t* scales,
                   const uint16_t* biases, const int32_t* idx, const float* scores, int T, int k,
                   int E, int I, int D, void* ws, size_t ws_bytes, uint16_t* y, void* stream);

/* SwiGLU with bf16 rounding after each op —
 * titan/adapters/mlx/vendor/mlx_lm/models/activations.py:9-11 with the gate/up
 * split of switch_layers.py:229-237.  gate_up [R, 2I] bf16 (gate columns
 * first) -> h [R, I] bf16 = silu(gate) * up. */
int tmoe_swiglu(const uint16_t* gate_up, int R, int I, uint16_t* h, void* stream);

/* ------------------------------------------------------------ weighted sum */

/* Unsort + routed weighted top-k sum — titan/kernels/moe_weighted_sum.py:163-195.
 * ys [T*k, D] bf16 in sorted order with inv_order [T*k] (flat -> sorted row),
 * or token-major when inv_order is NULL; scores [T, k] bf16; out [T, D] bf16.
 * mode 0 = clone (bit-identical to MLX's 8-partial bf16 reduce), 1 = fast. */
int tmoe_weighted_sum(const uint16_t* ys, const int32_t* inv_order, const uint16_t* scores, int T,
                      int k, int D, int mode, uint16_t* out, void* stream);

/* ------------------------------------------------------------- whole block */

/* One MoE layer's device weights (MLX layout) plus the prepared tables. */
typedef struct tmoe_layer {
  int hidden;           /* H */
  int num_experts;      /* E */
  int top_k;            /* k */
  int moe_inter;        /* I (expert intermediate) */
  int shared_inter;     /* Is (0: no shared expert) */
  const uint16_t* router_w;                                      /* [E, H] */
  const uint32_t* gate_up_w; const uint16_t* gate_up_s; const uint16_t* gate_up_b;  /* [E, 2I, .] */
  const uint32_t* down_w; const uint16_t* down_s; const uint16_t* down_b;           /* [E, H, .] */
  const uint16_t* gate_up_st; const uint16_t* gate_up_bt;        /* [E, H/64, 2I] */
  const uint16_t* down_st; const uint16_t* down_bt;              /* [E, I/64, H] */
  const uint32_t* shared_gate_up_w; const uint16_t* shared_gate_up_s;
  const uint16_t* shared_gate_up_b;                              /* [2Is, H/8], [2Is, H/64] */
  const uint32_t* shared_down_w; const uint16_t* shared_down_s;
  const uint16_t* shared_down_b;                                 /* [H, Is/8], [H, Is/64] */
  const uint16_t* shared_gate_up_st; const uint16_t* shared_gate_up_bt; /* [H/64, 2Is] */
  const uint16_t* shared_down_st; const uint16_t* shared_down_bt;       /* [Is/64, H] */
  const uint16_t* shared_gate_w;                                 /* [H] bf16 */
  /* Row normalisers of each projection, from tmoe_prepare_row_scale ([E, N]
   * fp32; NULL: that projection runs on the per-group kernels). */
  const float* gate_up_rs; const float* down_rs;
  const float* shared_gate_up_rs; const float* shared_down_rs;
} tmoe_layer;

typedef struct tmoe_options {
  int min_tokens;   /* T >= min_tokens: grouped-GEMM prefill path (default 512,
                       OMLX_MOE_INT8_MIN_TOKENS of patch.py:24-27); below it
                       the fp32 decode path */
  int down_int8;    /* 1: int8 down projection; 0: bf16-activation down
                       (OMLX_MOE_INT8_SKIP_DOWN=1) */
  int wsum_mode;    /* 0 clone, 1 fast */
  int int8_prefill; /* 1: int8 gate_up (the overlay installed); 0: the stock
                       bf16-activation grouped GEMMs for the prefill path */
  int gemm_kernel;  /* routed int8 prefill GEMMs: 0 = persistent TMA-fed tile
                       tcgen05 kernel (default; K <= 3072, else mma.sync),
                       1 = mma.sync (the comparison
                       baseline), 2 = persistent swap-AB tcgen05 kernel
                       (weight rows on the MMA's M side, TMA-fed; needs the
                       row normalisers).  All three keep the int8 algebra's
                       re-centred fp32 order bit for bit.  The
                       bf16-activation GEMMs (stock path, shared expert) run
                       on the swap-AB kernel whenever the layer carries its
                       row normalisers. */
  int decode_kernel; /* decode path (T < min_tokens): 0 = the whole layer in
                        one launch where the shape allows it (T <= 4, H, I
                        and Is multiples of 512), else 1 = router, gate_up
                        and down as three launches (always available) */
} tmoe_options;     /* NULL options = {512, 1, 0, 1, 0, 0} */

/* Device-side error record of the bounded waits inside the tcgen05 kernels
 * (no reference counterpart).  Synchronises the device; returns 0 when no
 * wait has timed out since the library was loaded, else TMOE_ERR_TIMEOUT. */
int tmoe_device_status(void);

/* Qwen3_5MoeSparseMoeBlock.__call__ —
 * titan/adapters/mlx/vendor/mlx_vlm/models/qwen3_5_moe/language.py:60-91 with
 * the int8 overlay installed.  x [T, H] bf16 -> y [T, H] bf16; idx_out [T, k]
 * int32 and scores_out [T, k] bf16 may be NULL.
 * The workspace must be zero-filled once, when it is allocated (its head holds
 * counters that every call leaves at zero again); reusing it across calls,
 * token counts and both paths needs no further clearing.  Calls sharing one
 * workspace must be ordered (one stream). */
size_t tmoe_moe_workspace_size(const tmoe_layer* layer, int T, const tmoe_options* opt);
int tmoe_moe_forward(const tmoe_layer* layer, const uint16_t* x, int T, const tmoe_options* opt,
                     void* ws, size_t ws_bytes, uint16_t* y, int32_t* idx_out,
                     uint16_t* scores_out, void* stream);

/* ------------------------------------------------ the decoder sub-layer */

/* RMSNorm with weight: out = bf16((x * r) * w), r = 1 / sqrt(mean(x^2) + eps)
 * in fp32 (the post-attention norm feeding the MoE block,
 * titan/adapters/mlx/vendor/mlx_vlm/models/qwen3_5_moe/language.py:103-107,137,
 * nn.RMSNorm).  x, out [T, H] bf16; weight [H] bf16. */
int tmoe_rmsnorm(const uint16_t* x, const uint16_t* weight, int T, int H, float eps, uint16_t* out,
                 void* stream);

/* Write a branch output back into the residual stream.  nstreams = 0: the
 * decoder layer's residual add out = bf16(residual + branch) [T, H]
 * (qwen3_5_moe/language.py:137).  nstreams = n > 0: the hyper-connection
 * inject into an n-wide stream, out[t, j] = bf16(residual[t, j] +
 * bf16(branch[t] * weights[t, j])), residual / out [T, n, H], weights [T, n]
 * bf16 (qwen4_exp/language.py:3198-3218, _hyper_inject). */
int tmoe_residual_inject(const uint16_t* branch, const uint16_t* residual, const uint16_t* weights,
                         int T, int H, int nstreams, uint16_t* out, void* stream);

/* The MoE sub-layer of a decoder layer in one call: the post-attention
 * RMSNorm of h, the block (tmoe_moe_forward), and the write-back:
 * nstreams = 0: out = h + block(norm(h)) (qwen3_5_moe/language.py:136-137);
 * nstreams = n: out = inject(residual [T, n, H], block(norm(h)), weights
 * [T, n]) (qwen4_exp/language.py:3338-3343).  The workspace follows
 * tmoe_moe_forward's rules (zero-filled once when allocated). */
size_t tmoe_moe_sublayer_workspace_size(const tmoe_layer* layer, int T, const tmoe_options* opt);
int tmoe_moe_sublayer(const tmoe_layer* layer, const uint16_t* norm_weight, float eps,
                      const uint16_t* h, int T, const uint16_t* residual,
                      const uint16_t* inject_weights, int nstreams, const tmoe_options* opt,
                      void* ws, size_t ws_bytes, uint16_t* out, void* stream);

/* Expert parallelism (no reference counterpart: the reference runs one
 * device).  Experts are sharded e // (E / W) over W ranks; these two calls are
 * the two halves of Qwen3_5MoeSparseMoeBlock.__call__ (language.py:74-91)
 * around the exchanges.
 *
 * Owner side: this rank's routed experts on rows received from other ranks.
 * `layer` describes the rank's E_local experts (router and shared-expert
 * fields unused).  x [R, H] bf16; pairs in row-major order: pair_row [P]
 * (received row), pair_exp [P] (local expert id).  y_pairs [P, H] bf16 gets
 * every pair's expert output, the same bits the single-device block computes
 * for that (token, slot). */
size_t tmoe_moe_experts_workspace_size(const tmoe_layer* layer, int R, int npairs,
                                       const tmoe_options* opt);
int tmoe_moe_experts(const tmoe_layer* layer, const uint16_t* x, int R, const int32_t* pair_row,
                     const int32_t* pair_exp, int npairs, const tmoe_options* opt, void* ws,
                     size_t ws_bytes, uint16_t* y_pairs, void* stream);

/* tmoe_moe_experts in slot form, for receive buffers of fixed capacity: pair
 * f = row*top_k + j of the R rows x [R, H] is served when slot_exp[f] >= 0
 * (its local expert; negative: skipped), and its output row is stored at
 * address y_rows[f] — in any device's memory that this one can write (the
 * expert-parallel return stores into the sources' buffers over NVLink from
 * the down GEMM's epilogue).  slot_exp [R*top_k] int32, y_rows [R*top_k]
 * device addresses; workspace tmoe_moe_experts_workspace_size(layer, R,
 * R*top_k, opt).  Every count stays on the device. */
int tmoe_moe_experts_slots(const tmoe_layer* layer, const uint16_t* x, int R,
                           const int32_t* slot_exp, const tmoe_options* opt, void* ws,
                           size_t ws_bytes, uint16_t* const* y_rows, void* stream);

/* Source side, before the exchanges: the token-local part of the layer on
 * this rank's tokens, with the kernels and arguments of tmoe_moe_forward's
 * grouped-GEMM path (language.py:74-84 and 85-90: the router Linear, softmax
 * top-k, the shared expert and its gate logit).  `layer` needs the router,
 * and the shared expert with its prepared tables when shared_inter > 0
 * (routed-expert fields unused).  idx [T, k] int32, scores [T, k] bf16;
 * gate_logit [T] fp32 and shared_out [T, H] bf16 when shared_inter > 0.
 * With these, the expert-parallel layer equals the single-device block bit
 * for bit on the int8 path, shared expert included. */
size_t tmoe_moe_local_workspace_size(const tmoe_layer* layer, int T, const tmoe_options* opt);
int tmoe_moe_local(const tmoe_layer* layer, const uint16_t* x, int T, const tmoe_options* opt,
                   void* ws, size_t ws_bytes, int32_t* idx, uint16_t* scores, float* gate_logit,
                   uint16_t* shared_out, void* stream);

/* Source side: the block's top-k weighted sum (moe_weighted_sum.py:142-195;
 * mode 0 clone, 1 fast) of every token's k expert outputs ys[inv[t*k+j]]
 * (inv NULL: ys[t*k+j], rows already token-major) plus the sigmoid-gated
 * shared expert (language.py:85-91; shared_out [T, D] bf16
 * and gate_logit [T] fp32, both NULL when there is none).  y [T, D] bf16. */
int tmoe_moe_combine(const uint16_t* ys, const int32_t* inv, const uint16_t* scores, int T, int k,
                     int D, int mode, const uint16_t* shared_out, const float* gate_logit,
                     uint16_t* y, void* stream);

/* ---- Expert-parallel exchanges over peer memory (no reference counterpart:
 * the reference runs one device).  Each rank allocates one exchange buffer,
 * maps every peer's through CUDA IPC, and passes `peers` (a DEVICE array of
 * world pointers, peers[rank] its own buffer) to dispatch and return.
 * Buffer layout for `world` ranks, `cap` tokens per source rank, k slots and
 * T_max tokens of its own; offsets[0..3] (bytes) locate:
 *   recv_x    [world][cap][H] bf16     rows sent to this rank by each source
 *   recv_meta [world][cap][k+1] int32  their k local expert ids (-1: not
 *                                      here), then the source token index
 *   ret       [T_max*k][H] bf16        expert output of this rank's pairs
 *   flags     [2][world] uint64        dispatch, return: epoch<<32 | count
 * Epochs start at 1 and grow by one per layer call; the buffer starts zeroed.
 * tmoe_ep_dispatch takes world + 1 zeroed device int32 counters and
 * leaves them zeroed.  Waits poll with a bounded back-off; on
 * timeout they write count -1 and tmoe_device_status returns
 * TMOE_ERR_TIMEOUT. */
size_t tmoe_ep_buffer_bytes(int world, int cap, int H, int k, int T_max, size_t* offsets);
int tmoe_ep_alloc(size_t bytes, void** ptr);
int tmoe_ep_free(void* ptr);
/* `handle` receives / supplies a cudaIpcMemHandle_t (64 bytes). */
int tmoe_ipc_handle(void* ptr, void* handle);
int tmoe_ipc_open(const void* handle, void** ptr);
int tmoe_ipc_close(void* ptr);
/* Source side: token t's row x[t] to every rank d owning one of idx[t, :]
 * (d = expert / experts_per_rank), at the next free row of this source's
 * recv_x block on d (rows land in no fixed order; the metadata row carries
 * the token index), then the number of rows sent posted in d's dispatch
 * flag.  counters: device int32 [world + 1], zeroed once; every call leaves
 * them zeroed. */
int tmoe_ep_dispatch(const uint16_t* x, const int32_t* idx, int T, int k, int H,
                     int experts_per_rank, int world, int rank, void* const* peers,
                     const size_t* offsets, int cap, int epoch, int32_t* counters, void* stream);
/* Waits for every peer's flag of `which` (0 dispatch, 1 return) at `epoch`
 * in the buffer `own`, writing the posted counts [world] (device int32). */
int tmoe_ep_wait(const void* own, const size_t* offsets, int which, int world, int epoch,
                 int32_t* counts, void* stream);
/* Owner side, after the dispatch wait: the slot form of the received rows
 * for tmoe_moe_experts_slots.  For f = (source * cap + i) * k + j,
 * slot_exp[f] is the local expert of slot j of received row i from that
 * source when the row was written this layer (i < rows_in[source], the
 * counts tmoe_ep_wait returned) and the expert is one of this rank's, else
 * -1; y_rows[f] is the address of the source's ret row token * k + j (NULL
 * where slot_exp is -1).  slot_exp [world*cap*k] int32, y_rows
 * [world*cap*k] device pointers. */
int tmoe_ep_slots(const void* own, const size_t* offsets, const int32_t* rows_in, int world,
                  int cap, int k, int experts_per_rank, int H, void* const* peers,
                  int32_t* slot_exp, uint16_t** y_rows, void* stream);

/* Posts (epoch, counts[d]) — count 0 when counts is NULL — in this rank's
 * slot of flag row `which` (0 dispatch, 1 return) of every rank d, after a
 * system-scope fence.  The owner side of the return: launched after
 * tmoe_moe_experts_slots has stored the sources' rows. */
int tmoe_ep_post(int which, const int32_t* counts, int world, int rank, void* const* peers,
                 const size_t* offsets, int epoch, void* stream);

/* The owner side of the return with failure propagation: as tmoe_ep_post(1,
 * NULL, ...), except that the count posted to every source is -1 when any
 * entry of rows_in [world] (the dispatch counts tmoe_ep_wait wrote) is
 * negative, i.e. when a dispatch wait of this layer gave up and this rank's
 * experts could not serve every row. */
int tmoe_ep_post_return(const int32_t* rows_in, int world, int rank, void* const* peers,
                        const size_t* offsets, int epoch, void* stream);

/* The source side after tmoe_moe_combine: when any of counts [world] (the
 * return counts tmoe_ep_wait wrote) is negative, the layer's output is not
 * valid; the call then records the error that tmoe_device_status reports and
 * overwrites y [n] (bf16) with NaN.  Otherwise it changes nothing. */
int tmoe_ep_guard(const int32_t* counts, int world, uint16_t* y, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TITAN_MOE_H */
