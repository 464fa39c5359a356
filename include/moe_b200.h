/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) fused FP8 block-scale MoE layer
 * moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no framework
 * types. All device pointers must live on the current CUDA device.
 *
 * Shapes (fixed by the operator definition, reference solution/cuda/kernel.h:8-23):
 *   H = 7168, I = 2048, E_global = 256, E_local = 32, top_k = 8,
 *   n_group = 8, topk_group = 4, block = 128.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_B200_API __attribute__((visibility("default")))
#else
#define MOE_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define MOE_B200_OK 0
#define MOE_B200_ERR_INVALID_ARGUMENT 1   /* null pointer, negative size, bad dtype code */
#define MOE_B200_ERR_MISALIGNED 2         /* a pointer breaks the alignment rule below */
#define MOE_B200_ERR_WORKSPACE_TOO_SMALL 3
#define MOE_B200_ERR_UNSUPPORTED_DEVICE 4 /* current device is not sm_100 */
#define MOE_B200_ERR_DRIVER 5             /* tensor-map encode unavailable or failed */
#define MOE_B200_ERR_CUDA 6               /* a CUDA runtime call failed */
#define MOE_B200_ERR_DEVICE_TIMEOUT 7     /* a kernel gave up a bounded wait */

#define MOE_B200_BIAS_BF16 0
#define MOE_B200_BIAS_FP32 1

/* Largest num_tokens accepted by the entry points below. */
#define MOE_B200_MAX_TOKENS 262144

/*
 * Bytes of device workspace moe_b200_run needs for num_tokens tokens.
 * The workspace is scratch owned by the caller; its contents need no
 * initialisation and are rewritten by every call.
 */
MOE_B200_API size_t moe_b200_workspace_bytes(int64_t num_tokens);

/*
 * Full MoE layer, destination-passing style: writes output[T, 7168] (bf16).
 *
 * Replaces the reference entry run(...) of solution/cuda/main.py:31-54 /
 * solution/cuda/main.cpp:13-142 (same arguments, same meaning), with the
 * output supplied by the caller as in the DPS form of the contest API
 * (reference README.md:227-257).
 *
 *   routing_logits        [T, 256]            fp32
 *   routing_bias          [256]               bf16 (bias_dtype 0) or fp32 (1)
 *   hidden_states         [T, 7168]           e4m3 (float8_e4m3fn bytes)
 *   hidden_states_scale   [56, T]             fp32, block-major
 *   gemm1_weights         [32, 4096, 7168]    e4m3; rows [0,2048) up, [2048,4096) gate
 *   gemm1_weights_scale   [32, 32, 56]        fp32
 *   gemm2_weights         [32, 7168, 2048]    e4m3
 *   gemm2_weights_scale   [32, 56, 16]        fp32
 *   local_expert_offset   first global expert id owned by this call
 *   routed_scaling_factor multiplies the renormalised routing weights
 *   output                [T, 7168]           bf16, written in full; may be NULL, then
 *                         the fp32 combine rows stay in the workspace (y_acc) for
 *                         moe_b200_ep_combine and no output is written
 *
 * Logits and bias must be finite. With a NaN among them the selection is
 * unspecified, but a token never selects the same expert twice.
 *
 * Alignment: hidden_states, gemm1_weights, gemm2_weights, routing_logits,
 * routing_bias and output 16 bytes; workspace 256 bytes.
 * The call is asynchronous on `stream` (a cudaStream_t) and performs no
 * host synchronisation, so it may be captured in a CUDA graph.
 */
MOE_B200_API int moe_b200_run(const float* routing_logits, const void* routing_bias, int routing_bias_dtype,
                 const void* hidden_states, const float* hidden_states_scale,
                 const void* gemm1_weights, const float* gemm1_weights_scale,
                 const void* gemm2_weights, const float* gemm2_weights_scale,
                 int64_t local_expert_offset, double routed_scaling_factor, int64_t num_tokens,
                 void* output, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The upstream quantiser of this operator's hidden states: bf16 [T, 7168]
 * -> e4m3 [T, 7168] and fp32 scales [56, T] (block-major, as moe_b200_run
 * reads them). Per 128-column block of a token row: scale = amax / 448
 * (1 for an all-zero block) and value = e4m3(x / scale), both divisions
 * IEEE fp32, rounded to nearest even and saturating. This is the
 * convention of the inputs the reference is benchmarked on; the reference
 * itself takes them pre-quantised (solution/cuda/main.py:31-42), so it has
 * no counterpart. Inputs must be finite. Alignment: hidden_states and
 * hidden_fp8 16 bytes, hidden_scale 4.
 */
MOE_B200_API int moe_b200_quantize_hidden(const void* hidden_states, int64_t num_tokens, void* hidden_fp8,
                                          float* hidden_scale, void* stream);

/*
 * moe_b200_run on bf16 hidden states [T, 7168] (no scale argument), with
 * the quantiser above inside the call: for T <= 64 it runs inside the copy
 * of each (token, expert) row into the permuted buffers (no e4m3 copy of
 * the hidden states is written); above, each token row is quantised once
 * into the workspace (hidden_q / hidden_qs of the layout) before routing.
 * Same result as moe_b200_quantize_hidden followed by moe_b200_run, and the
 * same workspace size. No reference counterpart (see above).
 */
MOE_B200_API int moe_b200_run_bf16_hidden(const float* routing_logits, const void* routing_bias,
                                          int routing_bias_dtype, const void* hidden_states,
                                          const void* gemm1_weights, const float* gemm1_weights_scale,
                                          const void* gemm2_weights, const float* gemm2_weights_scale,
                                          int64_t local_expert_offset, double routed_scaling_factor,
                                          int64_t num_tokens, void* output, void* workspace,
                                          size_t workspace_bytes, void* stream);

/*
 * Routing methods of this operator family, numbered as flashinfer's
 * RoutingMethodType. With l = logit + bias (bias optional except for
 * DeepSeek-V3) and k = top_k:
 *   DEFAULT            top-k of softmax(l), weight softmax(l)[e]
 *   RENORMALIZE        top-k of l, weights softmax of l over the k picks
 *   DEEPSEEK_V3        this operator's routing (moe_b200_run), k = 8
 *   LLAMA4             top-1 of l, weight sigmoid(l[e]); k = 1
 *   RENORMALIZE_NAIVE  top-k of softmax(l), weights renormalised over the picks
 *   TOPK               top-k of l, weights 1/k
 * every weight times routed_scaling_factor; ties go to the lower expert id.
 */
#define MOE_B200_ROUTING_DEFAULT 0
#define MOE_B200_ROUTING_RENORMALIZE 1
#define MOE_B200_ROUTING_DEEPSEEK_V3 2
#define MOE_B200_ROUTING_LLAMA4 3
#define MOE_B200_ROUTING_RENORMALIZE_NAIVE 4
#define MOE_B200_ROUTING_TOPK 5

/*
 * moe_b200_run with another routing method ahead of the same permutation,
 * GEMMs and combine (top_k 1..8; 8 for DEEPSEEK_V3, 1 for LLAMA4;
 * routing_bias may be NULL except for DEEPSEEK_V3). These are the sibling
 * definitions of the operator in flashinfer's MoE trace templates
 * (flashinfer/trace/templates/moe.py:187-390); the reference implements
 * only DeepSeek-V3 routing, so they have no reference counterpart.
 */
MOE_B200_API int moe_b200_run_routing(int routing_method, int top_k, const float* routing_logits,
                                      const void* routing_bias, int routing_bias_dtype,
                                      const void* hidden_states, const float* hidden_states_scale,
                                      const void* gemm1_weights, const float* gemm1_weights_scale,
                                      const void* gemm2_weights, const float* gemm2_weights_scale,
                                      int64_t local_expert_offset, double routed_scaling_factor,
                                      int64_t num_tokens, void* output, void* workspace,
                                      size_t workspace_bytes, void* stream);

/*
 * Routing only, any method above: topk_idx [T, 8] int32 global expert ids
 * best first, topk_w [T, 8] fp32; slots k >= top_k hold expert id
 * -(1 << 30) and weight 0.
 */
MOE_B200_API int moe_b200_route_method(int routing_method, int top_k, const float* routing_logits,
                                       const void* routing_bias, int routing_bias_dtype, int64_t num_tokens,
                                       double routed_scaling_factor, int32_t* topk_idx, float* topk_w,
                                       void* stream);

/*
 * Routing only: DeepSeek-V3 no-aux top-8 selection and weights.
 * Replaces the reference launcher launch_noaux_routing_topk8
 * (solution/cuda/kernel.h:37-44, kernel.cu:2527-2537). Experts are listed
 * best first (biased score descending, ties to the lower expert id).
 *   topk_idx [T, 8] int32 global expert ids, topk_w [T, 8] fp32.
 */
MOE_B200_API int moe_b200_route(const float* routing_logits, const void* routing_bias, int routing_bias_dtype,
                   int64_t num_tokens, double routed_scaling_factor, int32_t* topk_idx,
                   float* topk_w, void* stream);

/*
 * Reads the device status word of the last moe_b200_run that used this
 * workspace (synchronises `stream`). *status receives the raw bits (0 when
 * every bounded wait completed); returns MOE_B200_ERR_DEVICE_TIMEOUT when
 * any bit is set. Bits: 1 << 0..3 a GEMM role (TMA producer, MMA issuer,
 * epilogue, scale combiner) gave up a wait; 1 << 4 a routing pick out of
 * range; 1 << 5 a work-unit hand-off timed out; 1 << 6 a grid-wide arrival
 * count never completed; 1 << 7 an EP combine gave up waiting for a peer;
 * 1 << 8 an EP combine found its areas poisoned by an earlier give-up. The
 * word is cleared by each layer call. No reference counterpart (the
 * reference's waits are unbounded, solution/cuda/kernel.cu:300-307).
 */
MOE_B200_API int moe_b200_read_status(const void* workspace, uint32_t* status, void* stream);

/* Human-readable text for a status code. */
MOE_B200_API const char* moe_b200_status_string(int status);

/*
 * Byte offsets of the intermediate buffers inside the workspace, for
 * inspection by tests. No reference counterpart (the reference allocates
 * its intermediates per call, solution/cuda/main.cpp:50-108).
 */
typedef struct moe_b200_workspace_layout {
  size_t total_bytes;
  size_t counts;      /* int32[32] local-expert histogram */
  size_t status;      /* uint32 status word */
  size_t seg_off;     /* int32[33] expert segment starts (multiples of 16 rows) */
  size_t topk_idx;    /* int32[T, 8] */
  size_t topk_w;      /* fp32[T, 8] */
  size_t perm_tok;    /* int32[cap_rows] token of each permuted row, -1 for padding */
  size_t perm_w;      /* fp32[cap_rows] routing weight of each permuted row */
  size_t a_perm;      /* e4m3[cap_rows, 7168] token rows in permuted order */
  size_t sa_perm;     /* fp32[56, cap_rows] their block scales */
  size_t c_hi;        /* e4m3[cap_rows, 2048] */
  size_t c_lo;        /* e4m3[cap_rows, 2048] */
  size_t c_scale;     /* fp32[16, cap_rows] */
  size_t y_acc;       /* fp32[T, 7168] combine buffer (decode: row t = token t; otherwise
                         row tok_slot[t], the first n_touched rows in use) */
  size_t g1_acc;      /* fp32 K-split GEMM1 sums: [cap_rows, 4096] for T <= 64, [1664, 4096] for
                         T >= 512 (used when a batch has few token tiles); 0 for 64 < T < 512 */
  int64_t cap_rows;   /* round_up(8T, 16) + 32 * 16 + 128 */
  size_t chunk_counts; /* int32[ceil(T/256), 33] per-chunk expert counts + touched tokens */
  size_t sched;       /* int32[4] work-unit counters of the GEMM kernels */
  size_t perm_row;    /* int32[cap_rows] combine row of each permuted row, -1 in padding (not decode) */
  size_t tok_slot;    /* int32[T] combine row of each token, -1 without a local pick (not decode) */
  size_t n_touched;   /* int32 number of tokens with a local pick (not decode) */
  size_t slot_tok;    /* int32[T] token of each combine row, the first n_touched in use (not decode) */
  size_t hidden_q;    /* e4m3[T, 7168] quantised bf16 hidden states (moe_b200_run_bf16_hidden, not decode) */
  size_t hidden_qs;   /* fp32[56, T] their block scales (not decode) */
} moe_b200_workspace_layout;

MOE_B200_API int moe_b200_get_workspace_layout(int64_t num_tokens, moe_b200_workspace_layout* out);

/*
 * Profiling hook. When `events` is non-null, later moe_b200_run calls made
 * by the calling thread record events[i] (cudaEvent_t values created on the
 * current device) on their stream at the stage boundaries:
 *   0 start, 1 after the quantiser of bf16 hidden states (only
 *   moe_b200_run_bf16_hidden with more than 64 tokens runs one; otherwise
 *   nothing runs between 0 and 1), 2 after routing, 3 after the
 *   permutation, 4 after GEMM1 (+SwiGLU), 5 after GEMM2, 6 after the final
 *   bf16 conversion.
 * num_events must be 7. Pass NULL to switch the hook off. No reference
 * counterpart (the reference marks stages with NVTX ranges only,
 * solution/cuda/kernel.cu:477,1249,...).
 */
#define MOE_B200_NUM_STAGE_EVENTS 7
MOE_B200_API int moe_b200_set_stage_events(void* const* events, int num_events);

/*
 * Allocation-free variant of moe_b200_run for small batches. No counterpart
 * in the reference (its host code allocates per call, main.cpp:50-108).
 *
 * For callers that may not allocate device memory when they call the layer:
 * runtimes that reserve every buffer up front and forbid cudaMalloc later,
 * host code without a CUDA allocator to provide a workspace, or latency-
 * critical loops that cannot afford an allocation. The caller passes the
 * inputs and the output (same meaning and alignment as moe_b200_run); the
 * scratch is a fixed MOE_B200_NOALLOC_SCRATCH_BYTES array inside the library,
 * which every GPU that loads the library holds until the process exits.
 *
 * Limits and behaviour:
 *   - num_tokens <= MOE_B200_NOALLOC_MAX_TOKENS, otherwise the call returns
 *     MOE_B200_ERR_WORKSPACE_TOO_SMALL without doing anything;
 *   - the first call on a device looks up that device's array address (with
 *     the device current); make that first call before any stream capture;
 *   - all calls on a device share the one array: calls that may overlap on
 *     the GPU (different streams without ordering, or several threads) race
 *     and corrupt each other's results. Each call clears what must start at
 *     zero, so leftovers from the previous call do no harm;
 *   - no cudaMalloc, cudaFree or other allocating routine is called.
 */
#define MOE_B200_NOALLOC_MAX_TOKENS 16
#define MOE_B200_NOALLOC_SCRATCH_BYTES (24u << 20)
MOE_B200_API int moe_b200_run_noalloc(const float* routing_logits, const void* routing_bias,
                                      int routing_bias_dtype, const void* hidden_states,
                                      const float* hidden_states_scale, const void* gemm1_weights,
                                      const float* gemm1_weights_scale, const void* gemm2_weights,
                                      const float* gemm2_weights_scale, int64_t local_expert_offset,
                                      double routed_scaling_factor, int64_t num_tokens,
                                      void* output, void* stream);

/*
 * moe_b200_read_status for moe_b200_run_noalloc: reads the device status
 * word of the last allocation-free call on the current device (its status
 * word lives in the library's fixed array, which the caller cannot
 * address). Synchronises `stream`; same bits and return values as
 * moe_b200_read_status. A nonzero word means a kernel gave up a bounded
 * wait and the output of that call is not valid. Like the calls themselves,
 * it must not overlap another allocation-free call on the same device.
 */
MOE_B200_API int moe_b200_noalloc_read_status(uint32_t* status, void* stream);

/*
 * Expert-parallel combine over NVLink peer memory. No reference counterpart
 * (the reference is single-GPU).
 *
 * With expert parallelism every rank calls moe_b200_run on the same tokens
 * for its own expert shard (local_expert_offset) with output = NULL, on a
 * workspace that every rank can address (e.g. a moe_b200_ep_buffer_alloc
 * buffer mapped in every process through its IPC handle, below). Each rank
 * also owns an EP area of
 * moe_b200_ep_area_bytes(max tokens) bytes, equally addressable by all.
 * moe_b200_ep_combine then writes the bf16 sum over all ranks of the layer
 * output into `output` (this rank's, bf16 [T, 7168]): each rank reduces 1/W
 * of the token rows in fp32 from every rank's combine rows (peer loads),
 * rounds once to bf16 and stores the rows into every rank's area (peer
 * stores); the ranks synchronise through counters at the start of the areas.
 * Calls of at most 64 tokens instead exchange flagged lines (each 4-byte
 * value stored next to the call number, polled until the number matches):
 * every rank sends its partial sums of the rows another rank owns to that
 * rank, the owner adds the ranks' partial sums in rank order, rounds once
 * and sends the bf16 rows to every rank; no fence or counter is waited on.
 *
 *   rank_workspaces  host array of `world` pointers: rank q's workspace as
 *                    mapped in this process
 *   rank_areas       host array of `world` pointers: rank q's EP area
 *   rank, world      this rank and the number of ranks (<= 8)
 *
 * Every rank must call it once per layer call, on the stream of its
 * moe_b200_run, with the same num_tokens. Each EP area must be zero before
 * the first call; later calls need no clearing (the call number kept in the
 * area grows with every call, and each call's last CTA clears the per-call
 * counters itself). Each wait on a peer gives up after one second, sets
 * status bit 1 << 7 (moe_b200_read_status) and marks every rank's area as
 * poisoned: from then on every combine on those areas returns at once with
 * status bit 1 << 8 and writes no output. To recover, every rank
 * synchronises its device, zeroes its whole area (the counter block, the
 * first MOE_B200_EP_COUNTER_BYTES, and the flagged lines after it), and the
 * ranks meet at a host barrier before any of them calls the combine again.
 * Asynchronous, no host synchronisation.
 */
#define MOE_B200_EP_COUNTER_BYTES 256
MOE_B200_API size_t moe_b200_ep_area_bytes(int64_t num_tokens);
MOE_B200_API int moe_b200_ep_combine(void* const* rank_workspaces, void* const* rank_areas, int rank, int world,
                                     int64_t num_tokens, void* output, void* stream);

/*
 * moe_b200_ep_combine for ranks that own several 32-expert shards each (for
 * example all 8 shards of the 256 experts on fewer than 8 GPUs). Each rank
 * runs one moe_b200_run per shard with output = NULL, each on its own
 * workspace; shard_workspaces lists world * shards_per_rank workspaces,
 * rank-major (rank q's shards at [q * shards_per_rank, (q + 1) *
 * shards_per_rank)), as mapped in this process. The output is the bf16
 * rounding of an fp32 sum: each rank's shards summed in shard order, then
 * those sums added in rank order (with one shard per rank, the plain sum in
 * rank order).
 * world * shards_per_rank <= 8. The status word written is that of this
 * rank's first shard workspace. moe_b200_ep_combine is this call with
 * shards_per_rank = 1. No reference counterpart.
 */
MOE_B200_API int moe_b200_ep_combine_shards(void* const* shard_workspaces, int shards_per_rank,
                                            void* const* rank_areas, int rank, int world, int64_t num_tokens,
                                            void* output, void* stream);

/*
 * Device buffers that other processes of the node map through CUDA IPC, for
 * the workspaces and EP areas above: plain cudaMalloc memory (one allocation
 * per buffer, zero-filled, no multicast object), a 64-byte handle per
 * buffer, opened in a peer process with peer access enabled. Set-up calls:
 * alloc and open synchronise the device. No reference counterpart.
 */
#define MOE_B200_IPC_HANDLE_BYTES 64
MOE_B200_API int moe_b200_ep_buffer_alloc(size_t bytes, void** buffer);
MOE_B200_API int moe_b200_ep_buffer_free(void* buffer);
MOE_B200_API int moe_b200_ipc_get_handle(const void* buffer, void* handle);
MOE_B200_API int moe_b200_ipc_open_handle(const void* handle, void** buffer);
MOE_B200_API int moe_b200_ipc_close_handle(void* buffer);

/*
 * moe_b200_run with the routing given by the caller instead of computed:
 * topk_idx / topk_w are [T, top_k] (top_k 1..8) global expert ids and final
 * weights (no routed_scaling_factor is applied); ids outside
 * [local_expert_offset, local_expert_offset + 32) contribute nothing. The
 * permutation, GEMMs and combine are those of moe_b200_run, on the same
 * workspace size. Used on the rows an all-to-all dispatch delivered (below);
 * the reference has no counterpart (it always routes itself,
 * solution/cuda/main.cpp:50-57). Alignment: topk_idx and topk_w 4 bytes.
 * Its workspace is moe_b200_routed_workspace_bytes(T, top_k) bytes (a token
 * has at most top_k picks, so the permuted buffers are top_k / 8 of those of
 * moe_b200_run), laid out as moe_b200_get_routed_workspace_layout gives.
 */
MOE_B200_API size_t moe_b200_routed_workspace_bytes(int64_t num_tokens, int top_k);
MOE_B200_API int moe_b200_get_routed_workspace_layout(int64_t num_tokens, int top_k,
                                                      moe_b200_workspace_layout* out);
MOE_B200_API int moe_b200_run_routed(const int32_t* topk_idx, const float* topk_w, int top_k,
                                     const void* hidden_states, const float* hidden_states_scale,
                                     const void* gemm1_weights, const float* gemm1_weights_scale,
                                     const void* gemm2_weights, const float* gemm2_weights_scale,
                                     int64_t local_expert_offset, int64_t num_tokens, void* output,
                                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Token-parallel expert parallelism: every rank holds its own tokens and owns
 * shards_per_rank = 8 / world 32-expert shards (rank q owns global experts
 * [32 S q, 32 S (q + 1))). No reference counterpart (the reference is
 * single-GPU and has no all-to-all).
 *
 * Per rank, an area of moe_b200_a2a_area_bytes(max_tokens, recv_capacity)
 * bytes that every rank maps (e.g. moe_b200_ep_buffer_alloc + IPC handles),
 * zero before the first call; max_tokens and recv_capacity must be the same
 * on every rank, and so must the GPUs' SM counts (dispatch runs two CTAs per
 * SM, and each rank waits until every rank's CTAs have written into its
 * slab, counting them as world x its own grid). recv_capacity rows bound what one rank can receive (a row
 * per token that has a pick on it): world * max_tokens can never overflow.
 * One layer call, on every rank, on one stream:
 *   1. moe_b200_route on this rank's T tokens -> topk_idx, topk_w [T, 8];
 *   2. moe_b200_a2a_dispatch: every token is stored once into the receive
 *      slab of each rank it has a pick on (its e4m3 row, its 56 block scales
 *      and its 8 picks with only those on that rank kept, the others "no
 *      expert" with weight 0), rows ordered by (source rank, token);
 *   3. per owned shard s: moe_b200_run_routed(slab_idx, slab_w, 8, slab_rows,
 *      slab_scale, weights of s, 32 (S rank + s), recv_capacity, NULL,
 *      workspace of s, ...), with the slab offsets of moe_b200_a2a_get_layout
 *      (rows past the received count hold no pick) and workspaces of
 *      moe_b200_routed_workspace_bytes(recv_capacity, 8) bytes;
 *   4. moe_b200_a2a_combine: each own token's bf16 output is the fp32 sum of
 *      its combine rows on every shard of every rank it was sent to (each
 *      rank's shards in shard order, then the ranks in rank order), read from
 *      the owning ranks' workspaces (shard_workspaces: world * S,
 *      rank-major), rounded once.
 * Every rank must make all four steps for every call, also with T = 0. The
 * waits on peers give up after one second; then the area's status word gets
 * bit 1 << 7 and every rank's area is poisoned (bit 1 << 8 on later calls)
 * until each rank zeroes the first MOE_B200_A2A_COUNTER_BYTES of its area
 * after a device synchronisation and a host barrier. A slab too small for
 * what a rank received sets bit 1 << 9 (those picks are dropped).
 * moe_b200_a2a_read_status reads the status word and the received row count
 * (synchronises the stream).
 */
#define MOE_B200_A2A_COUNTER_BYTES 512
typedef struct moe_b200_a2a_layout {
  size_t total_bytes;
  size_t send_slot;   /* int32[max_tokens, 8] per destination rank: index of the token among this rank's tokens sent there, -1 if none */
  size_t dest_row;    /* int32[max_tokens, 8] per destination rank: the token's row in that rank's slab, -1 if none */
  size_t slab_idx;    /* int32[recv_capacity, 8] global expert ids of each received row's picks (none past the count) */
  size_t slab_w;      /* fp32[recv_capacity, 8] their routing weights */
  size_t slab_scale;  /* fp32[56, recv_capacity] block scales of the received rows */
  size_t slab_rows;   /* e4m3[recv_capacity, 7168] received token rows */
} moe_b200_a2a_layout;
MOE_B200_API size_t moe_b200_a2a_area_bytes(int64_t max_tokens, int64_t recv_capacity);
MOE_B200_API int moe_b200_a2a_get_layout(int64_t max_tokens, int64_t recv_capacity, moe_b200_a2a_layout* out);
MOE_B200_API int moe_b200_a2a_dispatch(const int32_t* topk_idx, const float* topk_w, const void* hidden_states,
                                       const float* hidden_states_scale, int64_t num_tokens, int64_t max_tokens,
                                       int64_t recv_capacity, void* const* rank_areas, int rank, int world,
                                       int shards_per_rank, void* stream);
MOE_B200_API int moe_b200_a2a_combine(const int32_t* topk_idx, void* const* shard_workspaces,
                                      void* const* rank_areas, int rank, int world, int shards_per_rank,
                                      int64_t num_tokens, int64_t max_tokens, int64_t recv_capacity,
                                      void* output, void* stream);
MOE_B200_API int moe_b200_a2a_read_status(const void* area, uint32_t* status, int32_t* recv_rows, void* stream);

/* ABI version of this header (bumped on any signature or struct layout change). */
MOE_B200_API int moe_b200_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
