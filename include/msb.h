/*
 * msb.h -- C ABI of the B200-native expert-indexed matmul over a GPU slot pool.
 *
 * This library replaces the hot path of MoEStream (monowalker/moestream):
 *   router expert ids -> ExpertCache remap to slot ids -> per-slot grouping
 *   -> ggml's GGML_OP_MUL_MAT_ID over a slab of quantized expert weights
 *   -> SwiGLU -> down projection -> router-weighted combine,
 * plus the slot fills that bring missing experts into the slab.
 *
 * Conventions (all entry points):
 *   - plain C types, opaque handles, `int` status return (MSB_OK == 0);
 *     msb_last_error() returns a thread-local message for the last failure;
 *   - no C++ exceptions cross this boundary;
 *   - every device pointer argument is memory on the device the handle lives on;
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy default
 *     stream. Kernels are stream-ordered; nothing here synchronizes the host
 *     unless the comment says so.
 *
 * Tensor layout vocabulary follows ggml: ne[0] is the fastest dimension.
 *   as  : expert weights [K (in), N (out), n_slot + 1]; slot n_slot is the
 *         zero slot (every weight 0, so any row routed there yields exactly 0);
 *   b   : activations [K, b_ne1, n_tok], b_ne1 is 1 (one vector per token,
 *         shared by its top_k rows) or top_k (one vector per (token, k));
 *   ids : int32 [top_k, n_tok], read with byte strides nb0 / nb1;
 *   res : float32 [N, top_k, n_tok], contiguous.
 */
#ifndef MSB_H
#define MSB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MSB_OK               0
#define MSB_ERR_INVALID      1   /* bad argument (shape, pointer, type)        */
#define MSB_ERR_CUDA         2   /* a CUDA runtime call failed                 */
#define MSB_ERR_NOMEM        3   /* device or pinned host allocation failed    */
#define MSB_ERR_UNSUPPORTED  4   /* valid request this build does not handle   */
#define MSB_ERR_TIMEOUT      5   /* a bounded device wait gave up              */
#define MSB_ERR_IO           6   /* a file could not be opened or read         */

/* ---- element types (values are ggml's enum ggml_type) ------------------ */
#define MSB_TYPE_F32     0
#define MSB_TYPE_F16     1
#define MSB_TYPE_IQ4_NL 20   /* 32 elements: fp16 d + 16 B nibbles (18 B)    */
#define MSB_TYPE_BF16   30
#define MSB_TYPE_MXFP4  39   /* 32 elements: e8m0 e + 16 B nibbles (17 B)    */

/* ---- expert roles of one MoE layer (reference: role 0 gate, 1 up, 2 down;
 *      src/llama-moestream.cpp:434-445 parse_name) ------------------------- */
#define MSB_ROLE_GATE 0
#define MSB_ROLE_UP   1
#define MSB_ROLE_DOWN 2

/* Null expert / unassigned slot marker (reference ExpertCache NO_SLOT,
 * src/expert_cache.hpp:109). */
#define MSB_NO_SLOT 0xFFFFFFFFu

/* ======================================================================== */
/* Library                                                                   */
/* ======================================================================== */

/* Version as 10000*major + 100*minor + patch. */
int msb_version(void);

/* Message for the last failure on the calling thread ("" if none). */
const char *msb_last_error(void);

/* Bytes of one expert in ggml's block layout (N rows of K elements), or -1
 * when K is not a multiple of 32 or the type is not a block type.
 * Replaces the per-(layer, role) `expert_bytes` the reference records in
 * register_slab (src/llama-moestream.cpp:1211-1225, SlabInfo :68-75). */
int64_t msb_expert_bytes(int wtype, int64_t K, int64_t N);

/* Slot count for a slab the way the reference sizes it:
 *   s = round(frac * n_expert), raised so that one micro-batch's expected
 *   union of experts fits with a 1.15 margin plus top_k, clamped to
 *   [8, n_expert]. The allocation is s + 1 (the zero slot).
 * Replaces moestream::slab_slots (src/llama-moestream.cpp:1017-1086) for the
 * plain-fraction mode; returns s (not s + 1), or 0 when n_expert <= 1. */
uint32_t msb_slab_slots(int64_t n_expert, double frac, int top_k, int max_ubatch);

/* Largest token count the slot pool can serve without exhausting it:
 * max n with n_expert*(1-(1-top_k/n_expert)^(n+1))*1.15 + top_k <= n_slot.
 * Batches above it take the full-arena path. Replaces the threshold in
 * finalize (src/llama-moestream.cpp:1530-1543). */
int msb_arena_threshold(int64_t n_expert, int top_k, uint32_t n_slot);

/* ======================================================================== */
/* Slot pool (device slab)                                                    */
/* ======================================================================== */

typedef struct msb_pool_s *msb_pool_t;

typedef struct {
  int      wtype;          /* MSB_TYPE_IQ4_NL or MSB_TYPE_MXFP4              */
  int64_t  K;              /* input features (row length), multiple of 32    */
  int64_t  N;              /* output features (rows)                         */
  int32_t  n_slot;         /* usable slots; slot n_slot is the zero slot     */
  int32_t  device;         /* CUDA device ordinal                            */
  int64_t  expert_bytes;   /* ggml bytes of one expert                       */
  int64_t  slot_stride;    /* device bytes between consecutive slots         */
  void    *data;           /* device base of slot 0                          */
} msb_pool_info_t;

/* Allocate a device slab of n_slot + 1 slots for experts of shape [K, N] and
 * zero-fill the zero slot. `max_fill_batch` experts can be staged per fill
 * call (0 picks 4). Replaces the slab allocation the patched loader makes
 * from slab_slots (src/apply.py:47-83) and ensure_zero_slot
 * (src/llama-moestream.cpp:1749-1792). Synchronous. */
int msb_pool_create(int wtype, int64_t K, int64_t N, int32_t n_slot,
                    int32_t max_fill_batch, msb_pool_t *out);
int msb_pool_destroy(msb_pool_t pool);
int msb_pool_get_info(msb_pool_t pool, msb_pool_info_t *out);

/* Copy n experts given in ggml block layout (host memory; pinned memory makes
 * the copies asynchronous) into `slots` of the pool, stream-ordered on
 * `stream`, converting them to the pool's device layout on the way.
 * Each src[i] points at expert_bytes bytes. Slot indices must be < n_slot.
 * Replaces the read loop of ms_remap_fn (src/llama-moestream.cpp:1954-2028):
 * do_read / run_reads_parallel (:1230-1263) plus ggml_backend_tensor_set. */
int msb_fill_slots_async(msb_pool_t pool, int32_t n, const int32_t *slots,
                         const void *const *src_host, void *stream);

/* Same, with the ggml-layout source already in device memory (no staging). */
int msb_fill_slots_from_device_async(msb_pool_t pool, int32_t n,
                                     const int32_t *slots,
                                     const void *const *src_dev, void *stream);

/* Copy slot `slot` back out in ggml block layout into device memory `dst`
 * (expert_bytes bytes). Used to check fills. */
int msb_read_slot_async(msb_pool_t pool, int32_t slot, void *dst_dev,
                        void *stream);

/* ======================================================================== */
/* Routing: remap + per-slot grouping (device)                               */
/* ======================================================================== */

/* Grouped routing of one mul_mat_id call, all device arrays, caller-owned.
 * n_pairs = n_tok * top_k; pair index i = t * top_k + k.               */
typedef struct {
  int32_t *slot_ids;  /* [n_pairs]     slot of pair i                     */
  int32_t *counts;    /* [n_slot + 1]  pairs per slot                     */
  int32_t *offsets;   /* [n_slot + 2]  exclusive scan of counts           */
  int32_t *rows;      /* [n_pairs]     pair indices grouped by slot, each
                                       group in increasing pair order     */
  int32_t *active;    /* [n_slot + 2]  active[0] = #slots with pairs,
                                       active[1..] = those slots ascending */
} msb_route_t;

/* Remap router ids to slot ids and group the (token, k) pairs per slot.
 *   ids_dev   : int32 expert ids, element (k, t) at byte k*nb0 + t*nb1
 *               (the reference reads ids with strides, :1900-1952, :2481);
 *   table_dev : int32 [n_expert] expert -> slot (negative or >= n_slot means
 *               not resident). NULL means ids already hold slot ids.
 *   Out-of-range ids and non-resident experts map to the zero slot n_slot,
 *   as the reference does for exhaustion and invalid ids (:1904-1928).
 * Bit-exact and deterministic. Replaces the ms_remap_fn output loop
 * (src/llama-moestream.cpp:1900-1952) and ggml's internal row grouping. */
int msb_remap_group(const int32_t *ids_dev, int64_t nb0, int64_t nb1,
                    int32_t top_k, int32_t n_tok,
                    const int32_t *table_dev, int32_t n_expert, int32_t n_slot,
                    const msb_route_t *route, void *stream);

/* ======================================================================== */
/* Router: top-k experts and weights per token (device)                      */
/* ======================================================================== */

#define MSB_ROUTER_SOFTMAX_TOPK 0  /* softmax over the k selected logits (gpt-oss;
                                      = softmax over all, renormalised)      */
#define MSB_ROUTER_SOFTMAX_ALL  1  /* softmax over all experts, the selected
                                      probabilities as they are             */

/* For each token t (row t of `logits`, n_expert values of type F32, F16 or
 * BF16, rows nb1 bytes apart): ids[t*top_k + j] = the expert with the j-th
 * largest logit (lower index first among equal logits; NaN counts as -inf)
 * and w[t*top_k + j] its weight. 1 <= top_k <= min(32, n_expert),
 * n_expert <= 1024. The ids feed msb_remap_group with nb0 = 4,
 * nb1 = 4 * top_k. The router of llama.cpp's MoE graph that produces the
 * ids the reference remaps (build_remap, src/llama-moestream.cpp:2555). */
int msb_router_topk(const void *logits_dev, int logits_type, int64_t nb1,
                    int32_t n_tok, int32_t n_expert, int32_t top_k, int mode,
                    int32_t *ids_dev, float *w_dev, void *stream);

/* ======================================================================== */
/* mul_mat_id                                                                 */
/* ======================================================================== */

/* Workspace bytes for msb_mul_mat_id / msb_moe_ffn with these shapes
 * (activation copies, intermediate results and, for batches of up to 8
 * (token, k) pairs, the partial sums of the tensor cores' split over K). */
int64_t msb_workspace_bytes(int64_t K_max, int32_t n_tok, int32_t top_k,
                            int32_t n_slot);

/* res[n, k, t] = sum_i dequant(as[:, n, slot(k,t)])[i] * b[i, k % b_ne1, t]
 * for a grouped route. b is f32 or bf16 with element (i, j, t) at
 * b + t*b_nb2 + j*b_nb1 + i*elem (byte strides). res is f32, contiguous.
 * The activations are quantized per 32-element block to int8 with an fp16
 * scale (ggml's q8_0 vec_dot form); products accumulate in int32 per block
 * and in f32 across blocks. Operator contract: ggml_mul_mat_id(ctx, as, b,
 * ids), call sites research/spikes/s0_slot_slab/main.c:148,
 * research/spikes/s6_arena_mulmatid/main.c:134. */
int msb_mul_mat_id(msb_pool_t pool, const void *b_dev, int b_type,
                   int64_t b_ne1, int64_t b_nb1, int64_t b_nb2,
                   const msb_route_t *route, int32_t top_k, int32_t n_tok,
                   float *res_dev, void *workspace, int64_t workspace_bytes,
                   void *stream);

/* msb_mul_mat_id for callers that cannot allocate device memory: code
 * running inside another runtime's allocator or memory hooks, where calling
 * cudaMalloc would re-enter them, and hosts whose device memory is all
 * reserved up front. Same arguments and result as msb_mul_mat_id, minus the
 * workspace: it uses a fixed 8 MiB device array inside this library
 * (msb_workspace_bytes(K, n_tok, top_k, n_slot) must not exceed 8 MiB,
 * e.g. K = 2880 at 64 tokens x top-4; larger requests return
 * MSB_ERR_INVALID). The pool's device must be current. The array is held
 * on every GPU that loads the library until exit and is shared by all calls
 * on a device, so calls that overlap on the GPU race on it. The first call
 * on a device looks up the array's device address; make it before any
 * stream capture on that device. No counterpart in the reference. */
int msb_mul_mat_id_noalloc(msb_pool_t pool, const void *b_dev, int b_type,
                           int64_t b_ne1, int64_t b_nb1, int64_t b_nb2,
                           const msb_route_t *route, int32_t top_k,
                           int32_t n_tok, float *res_dev, void *stream);

/* Status bits of the library's kernels on the current device: nonzero when
 * a kernel's bounded wait (the wait limit, one second by default; see
 * MSB_OPT_WAIT_LIMIT_US) gave up, in which case that kernel stopped early
 * and its outputs are incomplete. Tensor-core pipeline: 1 producer,
 * 2 accumulator release, 4 stage arrival, 8 accumulator arrival, 16 teardown
 * drain; expert-parallel exchange: 32 rows from the peers, 64 results from
 * the peers. Kernels only set bits; call after synchronizing the streams
 * that ran them. clear != 0 resets the word. No counterpart in the
 * reference (ggml's CPU matmul has no waits; its remap fails safe to the
 * zero slot instead, src/llama-moestream.cpp:1913-1928). */
int msb_device_status(int32_t *status, int32_t clear);

/* Synchronizes `stream` (the host blocks) and reports the device status
 * word: MSB_OK when every bounded wait completed, MSB_ERR_TIMEOUT (with a
 * message naming the waits) when one gave up; clear != 0 then resets the
 * word so that later calls report only new timeouts. */
int msb_stream_check(void *stream, int32_t clear);

/* ======================================================================== */
/* MoE FFN layer                                                              */
/* ======================================================================== */

/* One MoE FFN layer over grouped routing:
 *   g = mul_mat_id(gate, x), u = mul_mat_id(up, x), a = silu(g) * u,
 *   r = mul_mat_id(down, a), y[:, t] = sum_k w[k, t] * r[:, k, t].
 * gate and up may be the same pool with up_row0 = N_ff (a fused gate_up
 * tensor whose first N_ff rows are the gate); otherwise up_row0 = 0.
 * x: f32 or bf16 [K, 1, n_tok] (byte stride x_nb1 between tokens);
 * w: f32 [top_k, n_tok] router weights (contiguous), or NULL when top_k is
 * 1, in which case y = r (the expert outputs, no weighting);
 * y: f32 [K, n_tok].
 * act_dev (optional, may be NULL): f32 [N_ff, top_k, n_tok] receives a.
 * Rows routed to the zero slot contribute exactly 0. With router weights the
 * weighted sum runs in the down projection's epilogue (no separate combine
 * kernel), over k in increasing order with one f32 fused multiply-add per k,
 * so y does not depend on which CTA finishes last.
 * Composition restated from research/spikes/s1_real_expert_stream/main.c:
 * 186-209 and research/spikes/s4_sweep_math/main.c:89-92. */
int msb_moe_ffn(msb_pool_t gate, msb_pool_t up, int64_t up_row0,
                msb_pool_t down, const void *x_dev, int x_type, int64_t x_nb1,
                const msb_route_t *route, const float *w_dev, int32_t top_k,
                int32_t n_tok, float *y_dev, float *act_dev, void *workspace,
                int64_t workspace_bytes, void *stream);

/* The activation between the gate/up and down projections of
 * msb_moe_ffn_act. MSB_ACT_SILU: silu(g) * u (what msb_moe_ffn applies).
 * MSB_ACT_SWIGLU_OAI: gpt-oss's clamped form, x = min(g, limit),
 * y = clamp(u, -limit, limit), h = x * sigmoid(alpha * x) * (y + 1)
 * (llama.cpp's swiglu_oai, alpha 1.702 and limit 7 for gpt-oss; the
 * reference's spikes use plain SwiGLU and the reference itself leaves the
 * activation to llama.cpp). Expert biases: msb_moe_ffn_ex. */
#define MSB_ACT_SILU        0
#define MSB_ACT_SWIGLU_OAI  1
typedef struct {
  int   kind;
  float alpha;
  float limit;   /* > 0 for MSB_ACT_SWIGLU_OAI */
} msb_ffn_act_t;

/* msb_moe_ffn with the activation chosen by `act` (NULL: MSB_ACT_SILU). */
int msb_moe_ffn_act(msb_pool_t gate, msb_pool_t up, int64_t up_row0,
                    msb_pool_t down, const void *x_dev, int x_type,
                    int64_t x_nb1, const msb_route_t *route, const float *w_dev,
                    int32_t top_k, int32_t n_tok, float *y_dev, float *act_dev,
                    const msb_ffn_act_t *act, void *workspace,
                    int64_t workspace_bytes, void *stream);

/* Expert biases of one MoE FFN layer (gpt-oss's ffn_{gate,up,down}_exps.bias:
 * f32 [n_expert][rows] in device memory), indexed by the router's expert id
 * as llama.cpp's add_id does, so a bias follows its expert to whatever slot
 * the remap gives it (the reference rewrites only the ids passed to
 * mul_mat_id, src/apply.py:100-140, and leaves the bias lookup on the
 * expert ids). Each is added to the f32 matmul result of every pair not
 * routed to the zero slot (before the activation for gate and up, before
 * the router weighting for down); pairs routed to the zero slot stay exactly
 * 0, and ids outside [0, n_expert) add no bias. A NULL row pointer skips
 * that projection's bias. For a fused gate_up bias [n_expert][2 N_ff]:
 * gate_b = base, up_b = base + up_row0, both lds 2 N_ff. */
typedef struct {
  const float *gate_b, *up_b, *down_b;  /* row of expert e at ptr + e * ld  */
  int64_t gate_ld, up_ld, down_ld;      /* floats between experts' rows     */
  const int32_t *ids;                   /* router ids [top_k, n_tok] (device) */
  int64_t ids_nb0, ids_nb1;             /* byte strides of ids              */
  int32_t n_expert;
} msb_ffn_bias_t;

/* msb_moe_ffn_act with optional expert biases (NULL: none) and, with
 * accumulate != 0 (router weights required), y += the weighted sum instead
 * of y = it. Accumulation lets a batch run in two calls over two routes of
 * the same ids, each sending the other's experts to the zero slot: the
 * experts already resident first, the ones being filled on another stream
 * second (after an event of the fill), so the fill overlaps the first
 * call's grouped GEMM. The two-call y differs from one call's only in the
 * rounding of that last addition. */
int msb_moe_ffn_ex(msb_pool_t gate, msb_pool_t up, int64_t up_row0,
                   msb_pool_t down, const void *x_dev, int x_type,
                   int64_t x_nb1, const msb_route_t *route, const float *w_dev,
                   int32_t top_k, int32_t n_tok, float *y_dev, float *act_dev,
                   const msb_ffn_act_t *act, const msb_ffn_bias_t *bias,
                   int32_t accumulate, void *workspace, int64_t workspace_bytes,
                   void *stream);

/* ======================================================================== */
/* Expert parallelism (packing around the all-to-all exchanges)               */
/* ======================================================================== */

/* The reference is single-process and single-GPU; these have no counterpart
 * there. Experts are split evenly over n_rank GPUs (expert e lives on rank
 * e / n_local as local slot e % n_local).
 *
 * Packs this rank's (token, k) rows for an equal-split all-to-all: row of
 * pair p = t*top_k + k goes to block dest = ids[p] / n_local of the send
 * buffer at row dest*cap + (its rank among earlier pairs with that
 * destination). Row r's bf16 activations (K values) start at
 * send_x + r*send_nb1 and its local expert id (int32, -1 for unused rows) is
 * at send_e + r*send_e_nb (byte strides; the id may live in the same row as
 * the activations, so that one exchange carries both). pos (int32
 * [n_tok * top_k]) records each pair's row, -1 for invalid ids or rows
 * beyond cap. x is f32 or bf16 [n_tok, K] with byte stride x_nb1 between
 * tokens. */
int msb_ep_dispatch(const int32_t *ids_dev, const void *x_dev, int x_type,
                    int64_t x_nb1, int32_t top_k, int32_t n_tok, int64_t K,
                    int32_t n_local, int32_t n_rank, int32_t cap,
                    void *send_x_dev, int64_t send_nb1, int32_t *send_e_dev,
                    int64_t send_e_nb, int32_t *pos_dev, void *stream);

/* y[t, :] = sum_k w[t, k] * back[pos[t*top_k + k], :] (k ascending), where
 * back (f32 [n_rank * cap, K]) holds the expert outputs returned by the
 * reverse all-to-all. */
int msb_ep_combine(const float *back_dev, const int32_t *pos_dev,
                   const float *w_dev, int32_t top_k, int32_t n_tok, int64_t K,
                   float *y_dev, void *stream);

/* ---- Exchange over NVLink peer memory (no counterpart in the reference) --
 * Replaces the two all-to-alls above for ranks of one node whose GPUs reach
 * each other's memory. Each rank creates one exchange buffer
 * (msb_ep_buffer_bytes), shares its IPC handle with the other ranks (any
 * host channel) and opens theirs; msb_ep_peers_t lists every rank's buffer
 * as mapped on this rank (its own buffer for its own rank). Per layer:
 *   msb_ep_dispatch_peers  rows to the experts' ranks, written directly into
 *                          their buffers (block `rank`, msb_ep_dispatch's
 *                          row order; K bf16 then the int32 local expert id,
 *                          rows msb_ep_row_bytes(K) apart; unused rows -1)
 *   msb_ep_remap_group     waits until every rank's rows for this rank
 *                          arrived, then msb_remap_group of the received
 *                          ids (top_k 1, no table; -1 -> zero slot)
 *   ... local FFN over the received rows (buffer offset 0) ...
 *   msb_ep_return_peers    results back into the sources' buffers
 *                          (or both at once: msb_ep_moe_ffn_peers)
 *   msb_ep_combine_peers   waits until every result for this rank arrived
 *                          (f32 rows at offset msb_ep_yback_offset), then
 *                          msb_ep_combine
 * msb_ep_wait(phase) is the wait alone (0: rows, 1: results). All ranks
 * must make the same calls in the same order. A wait gives up after about a
 * second and sets status bit 32 (rows) or 64 (results) (msb_device_status).
 * The sequence counters live in the buffers, so the calls may be captured
 * in a CUDA graph and replayed. */
#define MSB_EP_MAX_RANKS 8
#define MSB_EP_HANDLE_BYTES 64

typedef struct {
  int32_t n_rank, rank, cap;       /* ranks, this rank, rows per block      */
  int64_t K;                       /* activation width, multiple of 4       */
  void *peer[MSB_EP_MAX_RANKS];    /* every rank's buffer as mapped here    */
} msb_ep_peers_t;

int64_t msb_ep_buffer_bytes(int32_t n_rank, int32_t cap, int64_t K);
int64_t msb_ep_row_bytes(int64_t K);
int64_t msb_ep_yback_offset(int32_t n_rank, int32_t cap, int64_t K);
int msb_ep_buffer_create(int64_t bytes, void **buf, void *ipc_handle);
int msb_ep_buffer_open(const void *ipc_handle, void **peer_buf);
int msb_ep_buffer_close(void *peer_buf);
int msb_ep_buffer_destroy(void *buf);
int msb_ep_dispatch_peers(const msb_ep_peers_t *peers, const int32_t *ids_dev,
                          const void *x_dev, int x_type, int64_t x_nb1,
                          int32_t top_k, int32_t n_tok, int32_t n_local,
                          int32_t *pos_dev, void *stream);
int msb_ep_return_peers(const msb_ep_peers_t *peers, const float *y_loc_dev,
                        void *stream);
int msb_ep_wait(const msb_ep_peers_t *peers, int32_t phase, void *stream);
int msb_ep_remap_group(const msb_ep_peers_t *peers, int32_t n_slot,
                       const msb_route_t *route, void *stream);
int msb_ep_combine_peers(const msb_ep_peers_t *peers, const int32_t *pos_dev,
                         const float *w_dev, int32_t top_k, int32_t n_tok,
                         float *y_dev, void *stream);
/* The local FFN over the received rows with the return fused in: the down
 * projection's epilogue stores every result row straight into its source
 * rank's buffer over NVLink and the kernel's last CTA raises the result
 * flags, replacing msb_moe_ffn + msb_ep_return_peers. MXFP4 pools of
 * tensor-core shapes only (MSB_ERR_UNSUPPORTED otherwise, nothing launched);
 * route from msb_ep_remap_group; workspace as msb_moe_ffn with
 * n_tok = n_rank * cap, top_k = 1. */
int msb_ep_moe_ffn_peers(const msb_ep_peers_t *peers, msb_pool_t gate,
                         msb_pool_t up, int64_t up_row0, msb_pool_t down,
                         const msb_route_t *route, void *workspace,
                         int64_t workspace_bytes, void *stream);

/* ======================================================================== */
/* Measurement hooks                                                          */
/* ======================================================================== */

/* Options (msb_set_option), process-wide.
 * MSB_OPT_MXFP4_PATH selects the arithmetic of MXFP4 mul_mat_id: 0 (default)
 * = tensor cores (tcgen05 block-scaled FP4, activations as four e2m1 terms
 * per 32-element block) wherever the shapes allow (K a multiple of 64; an up
 * view starting on a 32-row boundary), the CUDA-core path otherwise; 1 = the
 * CUDA-core path everywhere (int8 activations per 32-element block with an
 * fp16 scale, ggml's q8_0 form).
 * MSB_OPT_WAIT_LIMIT_US sets how long every bounded device wait (tensor-core
 * pipeline barriers, expert-parallel flags) spins before it gives up and
 * sets its status bit: 1 .. 60,000,000 microseconds, default 1,000,000. It
 * applies to launches set up after the call (a captured CUDA graph keeps the
 * limit it was captured with). */
#define MSB_OPT_MXFP4_PATH 1
#define MSB_OPT_WAIT_LIMIT_US 2
/* MSB_OPT_WIDE_PASSES: how many (token, k) pairs one tensor-core pass over a
 * weight tile serves. 0 (default) = 24 when the batch has at least 12 pairs
 * per slot it can reach (prompt-sized batches; one CTA per SM), else 8
 * (decode; two CTAs per SM); 1 = always 8; 2 = always 24 (except where K is
 * split over idle CTAs, batches of up to 8 pairs). The arithmetic is the
 * same either way. */
#define MSB_OPT_WIDE_PASSES 3
/* MSB_OPT_IQ4NL_PATH selects the arithmetic of IQ4_NL mul_mat_id: 0
 * (default) = tensor cores for batches with at least 4 pairs per slot they
 * can reach (weights dequantized to fp16 d * kvalue in shared memory,
 * activations rounded to fp16, f32 accumulation; K a multiple of 64, rows a
 * multiple of 8, gate/up views on 128-row boundaries), the CUDA-core path
 * (q8_0 form) otherwise; 1 = the CUDA-core path everywhere; 2 = the tensor
 * cores wherever the shapes allow. */
#define MSB_OPT_IQ4NL_PATH 4
int msb_set_option(int option, int value);

/* Kernels this library has launched in this process (all threads). */
uint64_t msb_kernel_launches(void);

/* Arms a one-shot timing of the next fused gate/up matmul that msb_moe_ffn
 * launches on the calling thread: `start` (a cudaEvent_t) is recorded on the
 * launch stream just before that kernel and `stop` just after it. */
void msb_time_next_gate_up(void *start, void *stop);

/* ======================================================================== */
/* Device quantizers (ggml block layout out)                                  */
/* ======================================================================== */

/* Quantize n_rows rows of K f32 values (row stride K) to ggml blocks.
 * MXFP4 follows ggml/gguf's quantizer (e = floor(log2(amax)) - 2 + 127,
 * nearest doubled-e2m1 value, first index on ties); IQ4_NL uses this
 * library's deterministic scale search (see oracle). */
int msb_quantize_rows(int wtype, const float *src_dev, int64_t n_rows,
                      int64_t K, void *dst_dev, void *stream);

/* ======================================================================== */
/* Host expert cache (S3-FIFO) -- the reference's ExpertCache                 */
/* ======================================================================== */

typedef struct msb_cache_s *msb_cache_t;

/* Field-for-field the reference ExpertCache::Config
 * (src/expert_cache.hpp:63-75). */
typedef struct {
  uint32_t n_layer;
  uint32_t n_expert;
  uint32_t n_slot;        /* 0 derives it from cache_frac                  */
  double   cache_frac;
  double   pin_ratio;
  double   small_ratio;
  uint32_t ghost_mult;
  int32_t  layer_quota_adapt;
  uint32_t quota_period;
  double   quota_eta;
  uint32_t quota_min;
} msb_cache_config_t;

/* Reference CacheStats (src/expert_cache.hpp:38-55), in declaration order. */
typedef struct {
  uint64_t hit, miss, hit_pinned, hit_small, hit_main, ghost_hit, admit,
      evict, bypass, promote, bytes_fetched;
} msb_cache_stats_t;

/* Origins (reference enum class Origin, src/expert_cache.hpp:29-34). */
#define MSB_ORIGIN_DEMAND        0
#define MSB_ORIGIN_PREFETCH_HIGH 1
#define MSB_ORIGIN_PREFETCH_LOW  2
#define MSB_ORIGIN_SWEEP         3

/* Fill `cfg` with the reference defaults (src/expert_cache.hpp:63-75). */
void msb_cache_config_default(msb_cache_config_t *cfg);
int  msb_cache_create(const msb_cache_config_t *cfg, msb_cache_t *out);
void msb_cache_destroy(msb_cache_t c);
/* ExpertCache::acquire (src/expert_cache.cpp:62-153): returns 1 on a hit,
 * 0 on a miss; *slot gets the slot or MSB_NO_SLOT. */
int  msb_cache_acquire(msb_cache_t c, uint32_t layer, uint32_t expert,
                       int origin, uint32_t *slot);
/* ExpertCache::mark_resident / release / end_step
 * (src/expert_cache.cpp:155-167, :228-231). */
void msb_cache_mark_resident(msb_cache_t c, uint32_t layer, uint32_t expert,
                             uint64_t nbytes);
void msb_cache_release(msb_cache_t c, uint32_t layer, uint32_t expert);
void msb_cache_end_step(msb_cache_t c);
/* ExpertCache::build_pinned (src/expert_cache.cpp:32-60); freq has
 * n_layer * n_expert entries. Ties in frequency pin the lower expert id. */
void msb_cache_build_pinned(msb_cache_t c, const uint32_t *freq, size_t n);
void msb_cache_get_stats(msb_cache_t c, msb_cache_stats_t *out);
uint32_t msb_cache_n_slot(msb_cache_t c);
uint32_t msb_cache_slot_of(msb_cache_t c, uint32_t layer, uint32_t expert);
/* Per-layer quotas (reference layer_quota()), n_layer entries. */
void msb_cache_layer_quota(msb_cache_t c, uint32_t *out);

/* ======================================================================== */
/* Slot streamer: ms_remap_fn's host half                                    */
/* ======================================================================== */

typedef struct msb_streamer_s *msb_streamer_t;

/* One ExpertCache per layer with n_layer = 1, pin_ratio 0 and quota
 * adaptation off, exactly as finalize builds them
 * (src/llama-moestream.cpp:1438-1447). Zero slot = n_slot. */
int  msb_streamer_create(uint32_t n_layer, uint32_t n_expert, uint32_t n_slot,
                         uint64_t expert_bytes_total, msb_streamer_t *out);
void msb_streamer_destroy(msb_streamer_t s);

/* The decode remap of one layer (ms_remap_fn, src/llama-moestream.cpp:
 * 1799-2105, core loop :1900-1952): releases the references this layer took
 * on its previous call (:1839-1852), then for each (t, k) in order acquires
 * the expert (Origin::Demand), writes its slot to out_slots[t*top_k + k]
 * (zero slot on exhaustion or out-of-range id), and appends each miss as
 * (expert, slot) in first-seen order. Host memory throughout.
 * miss_experts / miss_slots must hold n_tok*top_k entries.
 * table_out (optional, n_expert entries) receives expert -> slot after the
 * call, -1 for experts without a slot. */
int msb_streamer_remap(msb_streamer_t s, uint32_t layer, const int32_t *ids,
                       int64_t nb0, int64_t nb1, int32_t top_k, int32_t n_tok,
                       int32_t *out_slots, int32_t *n_miss,
                       int32_t *miss_experts, int32_t *miss_slots,
                       int32_t *table_out);
/* Summed stats over the layers plus the exhaustion count. */
int msb_streamer_stats(msb_streamer_t s, msb_cache_stats_t *out,
                       uint64_t *n_exhausted);

/* ======================================================================== */
/* GGUF expert source: slot fills read straight from the model file          */
/* ======================================================================== */

/* The reference reads expert bytes out of the GGUF the model came from
 * (src/llama-moestream.cpp:1230-1263 do_read / run_reads_parallel), opening
 * every shard of a split file "<base>-NNNNN-of-MMMMM.gguf" (:571-598,
 * :1455-1466), reading metadata integers by key suffix (:601-693) and
 * checking every expert tensor against its shard's size (:1478-1506). This
 * library parses the GGUF itself (format versions 2 and 3, little-endian). */
typedef struct msb_gguf_s *msb_gguf_t;

typedef struct {
  const char *name;     /* owned by the handle                               */
  int      type;        /* ggml type id                                      */
  int      n_dims;      /* 1..4                                              */
  int64_t  ne[4];       /* ne[0] fastest; unused dimensions are 1            */
  int32_t  shard;       /* file of a split GGUF (0-based)                    */
  uint64_t offset;      /* absolute byte offset of the data in that file     */
  int64_t  nbytes;      /* bytes of the whole tensor                         */
} msb_gguf_tensor_t;

/* Opens a GGUF (any shard's name of a split one opens all shards), parses
 * every header and checks that each tensor lies inside its file. Fails with
 * MSB_ERR_IO when a shard is missing, MSB_ERR_INVALID on a malformed header
 * or a tensor past the end of its file, MSB_ERR_UNSUPPORTED on another
 * format version or an unknown tensor type. A handle is not thread-safe. */
int msb_gguf_open(const char *path, msb_gguf_t *out);
/* Waits for the handle's staged copies, closes the files, frees it. */
int msb_gguf_close(msb_gguf_t g);
int32_t msb_gguf_shard_count(msb_gguf_t g);
int64_t msb_gguf_tensor_count(msb_gguf_t g);
int msb_gguf_tensor_info(msb_gguf_t g, int64_t index, msb_gguf_tensor_t *out);
/* Index of the tensor with this name, -1 if absent. */
int64_t msb_gguf_find_tensor(msb_gguf_t g, const char *name);
/* Index of "blk.<layer>.ffn_{gate,up,down}_exps.weight" (role MSB_ROLE_*),
 * a 3-D tensor [K, N, n_expert]; -1 if absent. The reference's expert
 * tensor naming (src/llama-moestream.cpp:434-445 parse_name). */
int64_t msb_gguf_expert_tensor(msb_gguf_t g, int32_t layer, int role);
/* First integer key of the first shard whose name ends in key_suffix (e.g.
 * ".expert_used_count", ".block_count", ".expert_count"); MSB_ERR_INVALID
 * when there is none. Replaces gguf_kv_int (src/llama-moestream.cpp:610-693). */
int msb_gguf_kv_int(msb_gguf_t g, const char *key_suffix, int64_t *value);
/* Bytes of one expert per layer and role summed over every expert tensor
 * with more than one expert: the cost of one slot across the model
 * (gguf_bytes_per_slot, src/llama-moestream.cpp:771-830). */
uint64_t msb_gguf_bytes_per_slot(msb_gguf_t g);
/* Reads experts[i] (ggml block layout, nbytes / ne[2] bytes each) of 3-D
 * tensor `tensor` into host memory dst_host[i], with up to n_threads
 * threads taking experts in turn. Synchronous; MSB_ERR_IO on a short read. */
int msb_gguf_read_experts(msb_gguf_t g, int64_t tensor, int32_t n,
                          const int32_t *experts, void *const *dst_host,
                          int32_t n_threads);
/* Reads experts[i] into pinned host memory owned by the handle and fills
 * slots[i] of `pool` from it (msb_fill_slots_async), stream-ordered on
 * `stream`. The tensor's type, K and N must be the pool's. The reads are
 * synchronous; the copies are not. Two staging halves are used in turn:
 * a call waits only for the copies of the call before the previous one.
 * Replaces the read-and-upload of ms_remap_fn
 * (src/llama-moestream.cpp:1954-2028). */
int msb_gguf_fill_slots_async(msb_gguf_t g, int64_t tensor, msb_pool_t pool,
                              int32_t n, const int32_t *experts,
                              const int32_t *slots, int32_t n_threads,
                              void *stream);

/* ======================================================================== */
/* Prefill arena on the device                                              */
/* ======================================================================== */

/* When a micro-batch's expert union exceeds the slots (msb_arena_threshold),
 * the reference runs mul_mat_id against a per-layer arena holding every
 * expert (prefill_exps, src/llama-moestream.cpp:2147-2155), loads into arena
 * il % n_buf only the experts the batch needs that it does not hold yet
 * (load_layer_arena :2167-2283), and loads the next layer in the background
 * with the previous pass's union of that layer as the hint (pf_kick
 * :2285-2317); what the hint missed is read once the ids are known.
 * Here each arena buffer is three pools (gate, up, down) with one slot per
 * expert (slot e holds expert e; slot n_expert is the zero slot), filled
 * from the GGUF; route the batch with msb_remap_group(ids, ..., table NULL,
 * n_slot = n_expert) and run the FFN over the pools msb_arena_ready gives.
 * All calls come from one thread; the background load is the library's. */
typedef struct msb_arena_s *msb_arena_t;

typedef struct {
  uint64_t loads;          /* loads that read something                     */
  uint64_t hits;           /* loads with nothing left to read               */
  uint64_t experts_asked;  /* n_expert per load (what a full read would be) */
  uint64_t experts_read;   /* experts actually read                         */
  uint64_t bytes_read;     /* expert bytes read, all roles                  */
} msb_arena_stats_t;

/* Opens the GGUF (its own handle) and sets up n_buf arena buffers on the
 * current device. Layers: <arch>.block_count, else the highest layer with
 * expert tensors. Pools are allocated on a buffer's first load, and again
 * when a layer's type or shape differs from the buffer's. */
int msb_arena_create(const char *gguf_path, int32_t n_buf, int32_t n_threads,
                     msb_arena_t *out);
/* Waits for the background load and every recorded use, frees it all. */
int msb_arena_destroy(msb_arena_t a);
int msb_arena_info(msb_arena_t a, int32_t *n_layer, int32_t *n_expert,
                   int32_t *n_buf);
/* Loads into buffer layer % n_buf the experts with need[e] != 0 (need NULL:
 * all) that it does not hold for this layer; forgets what it held when it
 * held another layer. Reads are synchronous, uploads ordered on `stream`
 * after the last use of the buffer (msb_arena_release). Joins a background
 * load first. */
int msb_arena_load(msb_arena_t a, int32_t layer, const uint8_t *need,
                   void *stream);
/* msb_arena_load on a background thread (hint as `need`), uploads on
 * `stream`; one in flight at a time; needs n_buf >= 2. */
int msb_arena_prefetch(msb_arena_t a, int32_t layer, const uint8_t *hint,
                       void *stream);
/* Joins the background load; returns its status. */
int msb_arena_wait(msb_arena_t a);
/* The pools holding `layer`, with compute_stream made to wait for their
 * uploads. Fails when the buffer holds another layer. */
int msb_arena_ready(msb_arena_t a, int32_t layer, void *compute_stream,
                    msb_pool_t *gate, msb_pool_t *up, msb_pool_t *down);
/* Marks the end of this layer's reads on compute_stream (the next load
 * into its buffer waits for it). */
int msb_arena_release(msb_arena_t a, int32_t layer, void *compute_stream);
/* Counters (joins the background load first). */
int msb_arena_stats(msb_arena_t a, msb_arena_stats_t *out);

/* ======================================================================== */
/* Device slot streamer: the decode remap without a host round trip          */
/* ======================================================================== */

/* The same decisions as msb_streamer_remap (one ExpertCache per layer as
 * the reference's finalize builds them, src/llama-moestream.cpp:1438-1447;
 * decode loop :1900-1952), made by a kernel from cache state kept in device
 * memory, with the miss queue (experts and slots, first-seen order) in
 * mapped pinned memory: the reference's stated fix for its per-layer
 * GPU<->CPU synchronisation. A fill kernel then copies the missed experts
 * from pinned host memory into their slots, so remap, fills, grouping and
 * the FFN are all stream-ordered launches that a CUDA graph can hold.
 * on_host != 0 keeps the state in host memory and runs the same decision
 * code on the calling thread (ids and slots are host pointers, no fills):
 * for checking on machines without a GPU. */
typedef struct msb_dstreamer_s *msb_dstreamer_t;

/* n_layer caches of n_expert experts over n_slot slots (slot n_slot is the
 * zero slot); at most max_pairs (token, k) pairs per call. */
int msb_dstreamer_create(uint32_t n_layer, uint32_t n_expert, uint32_t n_slot,
                         int32_t max_pairs, uint64_t expert_bytes_total,
                         int on_host, msb_dstreamer_t *out);
/* Synchronizes the device, frees everything. */
int msb_dstreamer_destroy(msb_dstreamer_t s);
/* One layer's remap: releases the layer's previous references, acquires
 * every (t, k) in order; out_slots[t*top_k + k] = slot, or n_slot for an
 * invalid id or on exhaustion (device memory; ids read with byte strides
 * nb0 between k, nb1 between tokens). The layer's miss queue is replaced. */
int msb_dstreamer_remap(msb_dstreamer_t s, uint32_t layer, const int32_t *ids,
                        int64_t nb0, int64_t nb1, int32_t top_k, int32_t n_tok,
                        int32_t *out_slots, void *stream);
/* Fills the slots of the layer's last misses in `pool` (n_slot slots, as
 * the streamer's) from `src`: expert e in ggml layout at
 * src + e * src_expert_stride, pinned host memory or device memory. Call
 * once per role (gate, up, down) with that role's pool and source. */
int msb_dstreamer_fill(msb_dstreamer_t s, uint32_t layer, msb_pool_t pool,
                       const void *src, int64_t src_expert_stride,
                       void *stream);
/* msb_dstreamer_fill for n_roles (1..3) pools at once (gate, up and down of
 * the layer, say): one launch whose CTAs interleave the roles' tiles. */
int msb_dstreamer_fill_roles(msb_dstreamer_t s, uint32_t layer, int32_t n_roles,
                             const msb_pool_t *pools, const void *const *srcs,
                             const int64_t *src_expert_strides, void *stream);
/* The layer's last miss queue, read from the mapped memory: valid once the
 * remap has completed (after a stream or event synchronize). experts and
 * slots may be NULL; otherwise they hold max_pairs entries. */
int msb_dstreamer_misses(msb_dstreamer_t s, uint32_t layer, int32_t *n_miss,
                         int32_t *experts, int32_t *slots);
/* expert -> slot of a layer (-1 without one), n_expert entries; waits for
 * the device (every stream) first. */
int msb_dstreamer_table(msb_dstreamer_t s, uint32_t layer, int32_t *table);
/* Counters summed over layers plus the exhaustion count; waits for the
 * device first. */
int msb_dstreamer_stats(msb_dstreamer_t s, msb_cache_stats_t *out,
                        uint64_t *n_exhausted);

#ifdef __cplusplus
}
#endif
#endif /* MSB_H */
