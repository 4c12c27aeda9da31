/*
 * muserve_moe.h — C ABI of the B200 (sm_100a) FP8 mixture-of-experts path.
 *
 * Every compute entry point takes raw device pointers, explicit sizes and a CUDA stream,
 * never allocates device memory, never synchronises the stream, and returns an int status
 * (MSV_OK == 0, negative on error; msv_last_error() gives the message).  Work is enqueued
 * on `stream` only, so a caller can capture the calls in a CUDA graph (a statement this
 * header does not extend to msv_ragged_moe_gemm_fp8_noalloc).  The exceptions are set-up and
 * checking calls: msv_ipc_* map and unmap another process's allocation (no stream), and
 * msv_check_device_error synchronises the stream it is given.
 *
 * Paths cited as `file:line` are in the reference project (xuguanghan/muserve); each entry
 * point names the reference interface it replaces.
 */
#ifndef MUSERVE_MOE_H
#define MUSERVE_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* msv_stream_t; /* same type as cudaStream_t */

enum msv_status {
  MSV_OK = 0,
  MSV_ERR_INVALID = -1,     /* bad size, null pointer, misalignment, bad dtype code */
  MSV_ERR_UNSUPPORTED = -2, /* valid request this build does not implement */
  MSV_ERR_CUDA = -3,        /* CUDA runtime / driver error (launch, attribute) */
  MSV_ERR_TIMEOUT = -4      /* a bounded device-side wait gave up (reported by msv_check_device_error) */
};

enum msv_dtype { MSV_F32 = 0, MSV_BF16 = 1, MSV_I32 = 2, MSV_I64 = 3, MSV_E4M3 = 4 };

/* Message of the last failed call on this host thread ("" when none). */
const char* msv_last_error(void);
/* ABI version: major*10000 + minor*100 + patch. */
int msv_version(void);

/*
 * Number of kernels this library has launched in this process (host-side count, one per
 * launch call; a CUDA-graph replay launches the captured kernels without counting again).
 */
unsigned long long msv_launch_count(void);

/*
 * Router: softmax over E fp32 logits, top-k, optional renormalisation of the k weights.
 *   replaces: muserve/model/qwen35_layer_v2.py:569-572 (softmax, torch.topk, /sum, .to(bf16))
 *             muserve/kernels/moe_dispatch.py:20-24 (moe_gate after the fp32 logits GEMM)
 * The selected ids and their order equal torch's CPU topk on the same values, ties included
 * (torch runs libstdc++ nth_element + sort, or partial_sort when k*64 <= E; this kernel
 * replays those algorithms, comparing logits, which order like the softmax scores).
 * logits: [T, ld_logits] fp32.  topk_w: [T,k] of w_dtype (MSV_F32 | MSV_BF16).
 * topk_ids: [T,k] of ids_dtype (MSV_I32 | MSV_I64).  1 <= k <= 16, k <= E <= 1024.
 */
int msv_route_topk(const float* logits, int64_t ld_logits, int T, int E, int k, int renormalize,
                   void* topk_w, int w_dtype, void* topk_ids, int ids_dtype, msv_stream_t stream);

/*
 * Router from the hidden states: logits = hidden @ gate_w^T on the tensor cores (bf16 x bf16,
 * fp32 accumulation), then softmax / top-k / renormalisation exactly as msv_route_topk.
 *   replaces: muserve/model/qwen35_layer_v2.py:567-572 (bf16_linear(hidden, gate_w).float(),
 *             softmax, topk, renormalise; pass round_logits_bf16 = 1) and
 *             muserve/kernels/moe_dispatch.py:8-24 (moe_gate: fp32 linear, softmax, topk,
 *             renormalise; pass round_logits_bf16 = 0)
 * hidden: [T,H] bf16 contiguous; gate_w: [E,H] bf16 contiguous; both 16-byte aligned.
 * H % 64 == 0, 16 <= E <= 1024, E % 16 == 0, 1 <= k <= 16.
 * round_logits_bf16: round each fp32 logit to bf16 before the softmax (the bf16 GEMM output).
 * logits_out: optional [T,E] fp32, 16-byte aligned: the logits the routing used.
 * workspace: >= msv_router_workspace_size(T, H, E) bytes, 256-byte aligned (fp32 partial sums
 * of the K splits, summed in split order by a separate kernel: deterministic).
 */
size_t msv_router_workspace_size(int T, int H, int E);
int msv_router_from_hidden(const void* hidden, const void* gate_w, int T, int H, int E, int k, int renormalize,
                           int round_logits_bf16, void* topk_w, int w_dtype, void* topk_ids, int ids_dtype,
                           float* logits_out, void* workspace, size_t workspace_bytes, msv_stream_t stream);

/*
 * msv_router_from_hidden with an additive prior on the logits: the routing reads
 * logits[t,e] + logit_bias[e] (fp32 add after the optional bf16 rounding); logits_out still
 * receives the GEMM's logits.  logit_bias: [E] fp32, not NULL.  The reference has no such
 * term; it carries the expert-popularity prior of the 60-layer stack benchmark (Zipf(1.2) log
 * probabilities added to the router logits).
 */
int msv_router_from_hidden_bias(const void* hidden, const void* gate_w, int T, int H, int E, int k, int renormalize,
                                int round_logits_bf16, const float* logit_bias, void* topk_w, int w_dtype,
                                void* topk_ids, int ids_dtype, float* logits_out, void* workspace,
                                size_t workspace_bytes, msv_stream_t stream);

/*
 * Gemma-style RMSNorm of the residual stream, with the residual add before it fused in.
 *   replaces: muserve/model/qwen35_layer_v2.py:59-62 (rms_norm_gemma) as the decoder layer
 *             calls it at :713-714 (x2 = rms_norm_gemma(h, post_attention_layernorm.weight)),
 *             and the residual add h_flat + moe_out at :715
 * h: [T,H] bf16, in/out.  add: [T,H] bf16 or NULL; when given, first h <- bf16(h + add).
 * weight: [H] bf16, stored as an offset from 1.0.  out: [T,H] bf16, or NULL to do the add only
 * (then add must be given).
 * out = bf16(h * rstd * bf16(1 + weight)), rstd = 1 / sqrt(mean(h^2) + eps), in fp32 with one
 * rounding, as torch's rms_norm on bf16.  H % 8 == 0, H <= 16384, pointers 16-byte aligned.
 */
int msv_add_rms_norm_gemma(void* h, const void* add, const void* weight, int T, int H, float eps, void* out,
                           msv_stream_t stream);

/*
 * Top-k selection only, on given fp32 values (no softmax): torch.topk(values, k) order.
 *   replaces: the torch.topk call of muserve/model/qwen35_layer_v2.py:570
 * out_values may be NULL.
 */
int msv_topk_select(const float* values, int64_t ld, int T, int E, int k, void* topk_ids, int ids_dtype,
                    float* out_values, msv_stream_t stream);

/*
 * Dispatch bookkeeping: filter the slots whose expert is local, stable-sort them by local
 * expert, pad the total to `alignment` rows with id -1.
 *   replaces: muserve/model/qwen35_layer_v2.py:574-605 (expand, local_mask, argsort(stable),
 *             inverse argsort, pad to 128)
 * topk_ids: [T,k] (ids_dtype MSV_I32 | MSV_I64).  Local experts: all E when placement==0
 * (TP=1 or intermediate-sharded experts), else e % tp == rank with local id e / tp
 * (muserve/loader.py:230-264).
 * Outputs (device): sort_order [T*k] int64 and inverse_order [T*k] int64 (first num_local
 * valid), sorted_expert_ids [ceil(T*k/alignment)*alignment] int32, expert_counts [E_local]
 * int32, num_local [1] int32.  Any output pointer may be NULL except num_local.
 */
int msv_moe_permute(const void* topk_ids, int ids_dtype, int T, int k, int num_experts, int placement,
                    int tp, int rank, int alignment, int64_t* sort_order, int64_t* inverse_order,
                    int32_t* sorted_expert_ids, int32_t* expert_counts, int32_t* num_local,
                    msv_stream_t stream);

/*
 * Per-row, per-128-channel e4m3 quantisation: s = max(amax|x|, 1e-12) / 448,
 * q = clamp(x / s, ±448) rounded to nearest even.
 *   replaces: muserve/model/qwen35_layer_v2.py:71-86 (_fast_fp8_quantize)
 * x: bf16 rows of length K (K % 128 == 0), row r read from x + src*ldx with
 * src = row_index ? row_index[r] : r (src < 0 leaves row r untouched).
 * q: [M, ldq] bytes; scale element (r, kb) at scale[r*s_row + kb*s_kb].
 */
int msv_fp8_quant_128(const void* x, int64_t ldx, int M, int K, const int32_t* row_index, uint8_t* q,
                      int64_t ldq, float* scale, int64_t s_row, int64_t s_kb, msv_stream_t stream);

/*
 * Ragged (row-grouped) block-scaled FP8 GEMM on tcgen05 tensor cores:
 *   out[m, n] = bf16( sum_kb (A[m,kb] . W[e_m, n, kb]) * a_scale[m,kb] * w_scale[e_m, n/128, kb] )
 * for rows with e_m = m_indices[m] >= 0; rows with -1 are left untouched.
 *   replaces: mate.gemm.ragged_m_moe_gemm_8bit((a, a_s), (w, w_s), m_indices, out)
 *             called at muserve/model/qwen35_layer_v2.py:613-618 and :638-643
 * a: [M,K] e4m3, a_scale: [M, K/128] f32, w: [E,N,K] e4m3, w_scale: [E, N/128, K/128] f32,
 * out: [M,N] bf16.  K % 128 == 0, N % 128 == 0.  Rows of one expert may be spread over
 * several runs.  workspace: msv_ragged_gemm_workspace_size(M, N) bytes (16-byte aligned).
 */
size_t msv_ragged_gemm_workspace_size(int M, int N);
int msv_ragged_moe_gemm_fp8(const uint8_t* a, const float* a_scale, int M, int K, const uint8_t* w,
                            const float* w_scale, int E, int N, const int32_t* m_indices, void* out,
                            void* workspace, size_t workspace_bytes, msv_stream_t stream);

/*
 * Allocation-free form of msv_ragged_moe_gemm_fp8: same arguments minus the workspace, same
 * kernels, same results.  It has no counterpart in the reference.
 *   Who needs it: callers that cannot hand the library device memory.  A serving engine that
 *   has given all free HBM to its KV-cache pool has none left for a per-call workspace; a host
 *   program that binds the reference's signature (which takes no workspace) over an FFI has
 *   no allocator it can call from that binding; a caller on a latency-critical decode loop
 *   cannot take the device-wide synchronisation that cudaFree implies.  This entry point
 *   calls no cudaMalloc, cudaFree or other allocating routine, on the device or (on success)
 *   the host.
 *   Scratch: a 4 MiB file-scope device array inside the library, one per device, holding the
 *   tile list.  Limit: M * (N/128) <= 262128 (e.g. M <= 8191 rows at N = 4096, M <= 32766 at
 *   N = 1024); larger sizes return MSV_ERR_INVALID with a message naming the limit.
 *   Set-up: the first call on a device, with that device current, looks up the array's device
 *   address (cudaGetSymbolAddress) and keeps it; make that first call before any stream
 *   capture on the device.
 *   Sharing: every call on one device uses the same array, which keeps the last call's tile
 *   list.  Calls that run in stream order are safe; calls that overlap on the GPU (different
 *   streams without ordering between them, or several host threads) race on the array.
 */
int msv_ragged_moe_gemm_fp8_noalloc(const uint8_t* a, const float* a_scale, int M, int K, const uint8_t* w,
                                    const float* w_scale, int E, int N, const int32_t* m_indices, void* out,
                                    msv_stream_t stream);

/*
 * Dense block-scaled FP8 GEMM, NT:  out[m,n] = bf16(sum_kb (a[m,kb].b[n,kb]) a_s[m,kb] b_s[n/128,kb]).
 *   replaces: mate.gemm.gemm_fp8_nt_groupwise(a, b, a_s, b_s, scale_granularity_mnk=(1,128,128),
 *             out_dtype=bf16) at muserve/model/qwen35_layer_v2.py:102-106, and
 *             muserve/kernels/fp8_matmul.py:172-216 (w8a8_block_fp8_matmul, block [128,128])
 * a [M,K] e4m3, a_scale [M,K/128] f32, b [N,K] e4m3, b_scale [N/128,K/128] f32, out [M,N] bf16.
 */
size_t msv_gemm_fp8_workspace_size(int M, int N);
int msv_gemm_fp8_nt_groupwise(const uint8_t* a, const float* a_scale, int M, int K, const uint8_t* b,
                              const float* b_scale, int N, void* out, void* workspace, size_t workspace_bytes,
                              msv_stream_t stream);

/* ── whole MoE layer ─────────────────────────────────────────────────────────────────── */

/* Rounding order of the weighted combine (which reference function's output to reproduce). */
enum msv_combine_mode {
  MSV_COMBINE_V2 = 0,       /* qwen35_layer_v2.py:660-662: bf16(w*d) per slot, fp32 sum over slots, one rounding */
  MSV_COMBINE_DISPATCH = 1, /* moe_dispatch.py:75-77: per expert ascending, out = bf16(out + d*w_fp32) */
  MSV_COMBINE_BATCHED = 2   /* batched_moe.py:153-158: per expert ascending, out = bf16(out + bf16(d*w)) */
};

typedef struct msv_moe_shape {
  int tokens;        /* T */
  int hidden;        /* H, multiple of 128 */
  int num_experts;   /* E (global) */
  int top_k;         /* k <= 16 */
  int inter;         /* routed intermediate held by this rank (I, or I/tp when sharded), multiple of 128 */
  int shared_inter;  /* shared-expert intermediate held by this rank; 0 = no shared expert */
  int placement;     /* 0: this rank holds every expert (TP=1 or intermediate-sharded);
                        1: this rank holds experts e % tp == rank (muserve/loader.py:232) */
  int tp;            /* tensor-parallel size (placement 1 only) */
  int rank;          /* tensor-parallel rank (placement 1 only) */
  int add_shared;    /* 1: add the shared expert on this rank (all ranks when its intermediate is sharded) */
  int combine_mode;  /* enum msv_combine_mode */
  int weights_dtype; /* topk weights input/output dtype for the combine: MSV_BF16 (V2) or MSV_F32 */
} msv_moe_shape;

typedef struct msv_moe_weights {
  /* routed experts, e4m3, K-major.  Expert e's gate rows start at row e*gu_expert_rows of
     gate_w, its up rows at row e*gu_expert_rows of up_w (a fused [E,2I,H] tensor is passed as
     gate_w = base, up_w = base + I*H, gu_expert_rows = 2I; separate tensors: gu_expert_rows = I). */
  const void* gate_w;
  const void* up_w;
  int64_t gu_expert_rows;
  const float* gate_s; /* 128x128 block scales, [n-block][k-block] per expert */
  const float* up_s;
  int64_t gu_scale_expert_stride; /* floats between consecutive experts' scale blocks */
  const void* down_w;             /* [E_local, H, inter] */
  const float* down_s;            /* [E_local, H/128, inter/128] */
  /* shared expert (used when shape.shared_inter > 0) */
  const void* sh_gate_w;          /* [shared_inter, H] */
  const void* sh_up_w;            /* [shared_inter, H] */
  const void* sh_down_w;          /* [H, shared_inter] */
  const float* sh_gate_s;
  const float* sh_up_s;
  const float* sh_down_s;
  const void* sh_gate_logit_w;    /* moe.shared_expert_gate.weight [1,H] bf16, or NULL */
} msv_moe_weights;

/*
 * One MoE layer from router logits to the [T,H] bf16 output (this rank's partial sum when
 * the layer is tensor-parallel; the caller all-reduces it).
 *   replaces: muserve/model/qwen35_layer_v2.py:561-675 (moe_forward) after the router GEMM
 *             (:568), muserve/kernels/moe_dispatch.py:27-79 (moe_experts_fp8, with
 *             topk given) and muserve/kernels/batched_moe.py:19-115
 * router_logits: [T,E] fp32 (may be NULL when topk_ids/topk_w are given as inputs:
 *   flags & MSV_FWD_ROUTING_GIVEN).  topk_w [T,k] (shape.weights_dtype) and topk_ids [T,k]
 *   int32 are outputs (or inputs with MSV_FWD_ROUTING_GIVEN); either may be NULL as outputs.
 * workspace: msv_moe_forward_workspace_size(shape) bytes, 256-byte aligned.
 */
#define MSV_FWD_ROUTING_GIVEN 1
size_t msv_moe_forward_workspace_size(const msv_moe_shape* shape);
int msv_moe_forward(const msv_moe_shape* shape, const msv_moe_weights* weights, const void* hidden,
                    const float* router_logits, void* topk_w, int32_t* topk_ids, void* out, int flags,
                    void* workspace, size_t workspace_bytes, msv_stream_t stream);

/*
 * msv_moe_forward that also records 7 CUDA events on `stream` (events: cudaEvent_t[7]): before
 * the router, the dispatch, the gather+quantise, the gate_up GEMM, the down GEMM and the
 * combine, and after the combine, so a caller can time each kernel on the launching stream.
 * NULL entries are skipped (each recorded event costs some device time between kernels).
 * Same work and results as msv_moe_forward (no reference counterpart: profiling hook).
 */
int msv_moe_forward_profiled(const msv_moe_shape* shape, const msv_moe_weights* weights, const void* hidden,
                             const float* router_logits, void* topk_w, int32_t* topk_ids, void* out, int flags,
                             void* workspace, size_t workspace_bytes, msv_stream_t stream, void* const* events);

/* ── tensor-parallel combine + all-reduce over NVLink peer memory ────────────────────── */

/*
 * CUDA IPC of one device allocation between the ranks' processes (one process per GPU).
 * msv_ipc_export: a handle (msv_ipc_handle_bytes() bytes) for the allocation that holds `ptr`,
 * and ptr's offset in it.  msv_ipc_import: another process's handle + offset -> a pointer
 * valid in this process (peer loads and stores over NVLink).  msv_ipc_close: unmap a pointer
 * msv_ipc_import returned.  (Set-up of msv_moe_forward_tp; no reference counterpart.)
 */
size_t msv_ipc_handle_bytes(void);
int msv_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
int msv_ipc_import(const void* handle, uint64_t offset, void** ptr_out);
int msv_ipc_close(void* ptr);

#define MSV_MAX_TP 8

/*
 * The TP group of msv_moe_forward_tp.  Every rank allocates one shared buffer of
 * msv_tp_shared_bytes(max_tokens, hidden) bytes (256-byte aligned, zero-filled: its words carry
 * flags) and one epoch buffer of msv_tp_epoch_bytes() bytes (zero-filled), exports the shared
 * buffer and imports every other rank's.  shared[p] is rank p's buffer as mapped in this
 * process (shared[rank] is the local one).  After a MSV_ERR_TIMEOUT the buffers must be
 * zero-filled again on every rank before the next call.  Calls on one group may change the
 * token count (up to max_tokens) and the combine mode freely: the kernel's grid cap depends
 * only on the device and `hidden`, so each token keeps its CTA (and that CTA's flag counter)
 * from call to call.
 */
typedef struct msv_tp_comm {
  int world;                     /* ranks in the group, 1..MSV_MAX_TP */
  int rank;                      /* this rank */
  int max_tokens;                /* tokens each shared buffer holds */
  int hidden;                    /* H the shared buffers were sized for */
  void* shared[MSV_MAX_TP];
  unsigned int* epoch;
} msv_tp_comm;

size_t msv_tp_shared_bytes(int max_tokens, int hidden);
size_t msv_tp_epoch_bytes(void);

/*
 * msv_moe_forward with the weighted combine fused with the sum over the TP group: every rank
 * passes its shard of the layer (shape.inter = I/tp with placement 0, or placement 1), and
 * `out` receives the all-reduced [T,H] bf16 result, identical on every rank.
 *   replaces: muserve/model/qwen35_layer_v2.py:657-662 with muserve/distributed.py:62-64
 *             (the per-rank result, then all_reduce(SUM) over the TP group)
 * The partials are summed in fp32 in rank order and rounded to bf16 once.  A persistent grid
 * no larger than the SMs hold at once (at most T CTAs) combines the tokens and pushes each H/world-column slice to the rank that
 * owns it (peer stores of 8-byte words: two bf16 values and a flag); the owner sums the slices
 * and pushes the result to every rank, which copies its rows to `out`.  Waits are bounded
 * (MSV_ERR_TIMEOUT through msv_check_device_error).  T <= comm->max_tokens,
 * H == comm->hidden, H % (8 * world) == 0.  Every rank must make the same calls in the same
 * order on the same number of SMs.
 */
int msv_moe_forward_tp(const msv_moe_shape* shape, const msv_moe_weights* weights, const void* hidden,
                       const float* router_logits, void* topk_w, int32_t* topk_ids, void* out, int flags,
                       void* workspace, size_t workspace_bytes, const msv_tp_comm* comm, msv_stream_t stream);
/* msv_moe_forward_tp with the 7 events of msv_moe_forward_profiled (the last stage is the
   fused combine + all-reduce). */
int msv_moe_forward_tp_profiled(const msv_moe_shape* shape, const msv_moe_weights* weights, const void* hidden,
                                const float* router_logits, void* topk_w, int32_t* topk_ids, void* out, int flags,
                                void* workspace, size_t workspace_bytes, const msv_tp_comm* comm,
                                msv_stream_t stream, void* const* events);

/*
 * Reads and clears the device error word that the layer's kernels raise when a bounded wait
 * gives up.  Synchronises `stream`.  Returns MSV_OK or MSV_ERR_TIMEOUT.
 */
int msv_check_device_error(msv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MUSERVE_MOE_H */
