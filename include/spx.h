/*
 * libspx — B200 (sm_100a) kernels for SPALMER's routed micro-expert channel
 * mixer, behind a plain C ABI.
 *
 * All pointers are device pointers unless stated otherwise; BF16 tensors are
 * passed as uint16_t bit patterns; every tensor is contiguous row-major and
 * 16-byte aligned.  `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Every entry point returns SPX_OK (0) or a negative status; no C++
 * exception crosses this boundary.  The caller owns all memory: weights,
 * outputs and the workspace (size from spx_layer_sizes, zero-filled once
 * before first use).  Calls on distinct streams with distinct workspaces are
 * independent.
 *
 * Reference interfaces replaced (mESmaC/spalmer, paths under src/spalmer/):
 *   spx_layer_forward  MicroExpertChannelMixer.forward   experts/mixer.py:145-241
 *   spx_route          SurpriseRouter.forward (score transform, router.py:52-56)
 *                      + select_least_surprised_experts  experts/router.py:59-95
 *   spx_dispatch       _pair_counts / cumsum / argsort(stable=True)
 *                                                        experts/bank.py:721-723
 *   spx_pack_weights   derived cache of the state_dict layout
 *                                                        experts/bank.py:52-54, nn/ffn.py:16-18
 *   spx_softplus_table F.softplus on every BF16 input    experts/router.py:56
 *   spx_pack_weights_mxfp8  MXFP8 packing of the expert masters (the weight side
 *                      of _mxfp8_mm_nt)                  experts/native.py:113-140
 *   spx_mxfp8_quantize_rows _mx_quantize_rows (MXTensor.to_mx, E4M3, block 32,
 *                      RCEIL)                            experts/native.py:91-110
 *   spx_mxfp8_mm_nt    _mxfp8_mm_nt (left @ right_rows.T, both MXFP8, BF16 out)
 *                                                        experts/native.py:113-140
 *
 * Stage entry points (expert parallelism: the caller moves rows between GPUs
 * with NCCL all-to-all between them; on one GPU they compose to
 * spx_layer_forward):
 *   spx_layer_route    router + selection + dispatch     experts/mixer.py:176-199,
 *                                                        bank.py:721-736
 *   spx_gather_rows    hidden_states[token_index] in dispatch order   bank.py:751
 *   spx_swiglu_backward_rows  SwiGLU backward of rows (shared expert in the
 *                      layer's training step)            nn/ffn.py:27-30 (autograd)
 *   spx_experts_forward grouped expert SwiGLU of rows with given expert ids
 *                      (unweighted)                      bank.py:740-763
 *   spx_shared_forward SwiGLU.forward                    nn/ffn.py:27-30
 *   spx_combine        _weighted_expert_updates + index_add + shared add
 *                                                        bank.py:764-778, mixer.py:207
 *   spx_surprise_calibration  _attach_surprise_telemetry + _attribute_nll_to_experts
 *                                                        modeling.py:1468-1534
 */
#ifndef SPX_H_
#define SPX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPX_ABI_VERSION 12

#define SPX_OK 0
#define SPX_ERR_INVALID_ARG -1
#define SPX_ERR_UNSUPPORTED -2
#define SPX_ERR_CUDA -3
#define SPX_ERR_DRIVER -4
#define SPX_ERR_TIMEOUT -5
#define SPX_ERR_ALIGNMENT -6
#define SPX_ERR_WORKSPACE -7
#define SPX_ERR_DEVICE -8
#define SPX_ERR_SCRATCH_LIMIT -9 /* problem larger than spx_dispatch_static's fixed scratch */

/* Shape of one mixer layer (MicroExpertsConfig resolved values, experts/config.py:86-110,231-244). */
typedef struct spx_layer_dims {
  int64_t tokens;          /* T = batch * seq_len                               */
  int32_t d_model;         /* d                                                  */
  int32_t num_experts;     /* E (<= 1024)                                        */
  int32_t inter_dim;       /* I, resolved_inter_dim                              */
  int32_t shared_dim;      /* S, resolved_shared_inter_dim; 0 = no shared path   */
  int32_t top_k;           /* k, active experts per token (1..20, <= E)          */
  int32_t score_transform; /* 0 = softplus, 1 = identity (router_score_transform) */
  int32_t execution_loop;  /* 1 = telemetry of expert_execution="loop"          */
  int32_t mxfp8_lane;      /* low-precision lane of the layer (I % 32 == 0): 0 none,
                              1 = some experts may run ("mxfp8", "mxfp8"),
                              2 = some experts may run ("nvfp4", "nvfp4"); the
                              workspace then holds quantised activations     */
} spx_layer_dims;

/* The reference state_dict tensors (BF16), unchanged layouts. */
typedef struct spx_reference_weights {
  const uint16_t* router_weight; /* router.proj.weight            [E, d]    */
  const uint16_t* router_bias;   /* router.proj.bias              [E] | NULL */
  const uint16_t* gate_proj;     /* experts.gate_proj             [E, d, I] */
  const uint16_t* up_proj;       /* experts.up_proj               [E, d, I] */
  const uint16_t* down_proj;     /* experts.down_proj             [E, I, d] */
  const uint16_t* shared_gate;   /* shared.gate_projection.weight [S, d] | NULL */
  const uint16_t* shared_up;     /* shared.up_projection.weight   [S, d] | NULL */
  const uint16_t* shared_down;   /* shared.down_projection.weight [d, S] | NULL */
} spx_reference_weights;

/* Element counts (uint16_t) of the packed weight buffers; the *_mx fields
 * are BYTES of the MXFP8 copies (zero unless dims->mxfp8_lane).  Packed
 * layouts depend on the batch class of dims->tokens (<= 256 tokens: decode
 * tiles; more: throughput tiles): pack with a dims of the same class as the
 * forward that uses the weights. */
typedef struct spx_packed_sizes {
  size_t router_weight;
  size_t expert_w1;
  size_t expert_w2;
  size_t shared_w1;
  size_t shared_w2;
  size_t expert_w1_mx;        /* E4M3 [E, 2I, round_up(d, 128)]                  */
  size_t expert_w1_mx_scales; /* E8M0 scale atoms of expert_w1_mx                */
  size_t expert_w2_mx;        /* E4M3 [E, d, round_up(I, 128)]                   */
  size_t expert_w2_mx_scales; /* E8M0 scale atoms of expert_w2_mx                */
  size_t expert_nvfp4_amax;   /* bytes of the per-expert weight amax (NVFP4 lane) */
} spx_packed_sizes;

typedef struct spx_packed_weights {
  const uint16_t* router_weight;  /* from spx_pack_weights                     */
  const uint16_t* router_bias;    /* [E] | NULL                                */
  const uint16_t* expert_w1;
  const uint16_t* expert_w2;
  const uint16_t* shared_w1;      /* NULL when shared_dim == 0                 */
  const uint16_t* shared_w2;
  const uint16_t* softplus_table; /* [65536]; required for score_transform 0   */
  const uint8_t* resident_mask;   /* [E] (0/1) | NULL = full pool              */
  /* MXFP8 lane (dims->mxfp8_lane): per-expert kernel lane and the copies made
   * by spx_pack_weights_mxfp8.  expert_lane_mxfp8[e] = 1 runs expert e as
   * ("mxfp8", "mxfp8") -- MicroExpertBank._execution_pair, experts/bank.py:462-475. */
  const uint8_t* expert_lane_mxfp8; /* [E] (0/1) | NULL = every expert BF16 */
  const uint8_t* expert_w1_mx;
  const uint8_t* expert_w1_mx_scales;
  const uint8_t* expert_w2_mx;
  const uint8_t* expert_w2_mx_scales;
  /* NVFP4 lane (dims->mxfp8_lane == 2): the *_mx fields hold the copies made by
   * spx_pack_weights_nvfp4 (E2M1 values and UE4M3 scale atoms) and this the
   * per-expert amax of gate, up, down ([E][4] float, the 4th unused). */
  const float* expert_nvfp4_amax;
  /* [E] float reconstruction error of each expert's low-precision copies
   * (spx_expert_quant_error), or NULL: the forward then reports zeros, as the
   * reference does for bfloat16 / float32 expert weights. */
  const float* expert_quant_error;
} spx_packed_weights;

typedef struct spx_layer_outputs {
  uint16_t* update;                /* [T, d]  routed + shared update (required) */
  uint16_t* router_scores;         /* [T, E]  (required)                        */
  int64_t* expert_ids;             /* [T, k]  (required)                        */
  uint16_t* routing_weights;       /* [T, k]  (required)                        */
  float* expert_utilization;       /* [E]     | NULL                            */
  int64_t* group_stats;            /* [6] count, max_load, real, padded,
                                      counterfactual padded, num_active | NULL  */
  float* group_ratios;             /* [2] padding amplification,
                                      counterfactual amplification | NULL       */
  uint16_t* auxiliary_loss;        /* [1] BF16 load-balance loss | NULL         */
  int32_t* dispatch_order;         /* [T*k] argsort(stable) | NULL              */
  int32_t* expert_counts;          /* [E] | NULL                                */
  const uint16_t* injected_logits; /* [T, E] use instead of the router GEMM | NULL */
  uint16_t* router_logits;         /* [T, E] receives router GEMM output | NULL */
  void* const* stage_events;       /* NULL, or SPX_STAGE_EVENTS cudaEvent_t handles recorded
                                      on `stream` at the stage boundaries below            */
  int32_t* pair_rank;              /* [T*k] sorted position of each pair (inverse of
                                      dispatch_order) | NULL; required by spx_layer_route  */
  float* expert_quantization_error; /* [E] weights->expert_quant_error of the selected
                                      experts, 0 for the others | NULL (bank.py:526-566)   */
  /* Training (BF16 experts): activations for spx_layer_backward, written by
   * the expert GEMM1 from the rows it stages anyway, so the backward need
   * not recompute it.  Both or neither; with them the expert projections
   * always run as tcgen05 GEMMs (no decode GEMVs).                          */
  uint16_t* saved_x;               /* [T*k, d] hidden rows in dispatch order | NULL  */
  uint16_t* saved_gu;              /* [T*k, spx_layer_saved_gu_cols] gate | up pre-
                                      activations (BF16) in dispatch order | NULL   */
  uint16_t* saved_shared_gu;       /* [T, cols of spx_layer_saved_shared_gu] the shared
                                      SwiGLU's gate | up pre-activations (BF16), per
                                      chunk of `chunk` columns its gate then its up
                                      columns | NULL (the shared SwiGLU's backward
                                      input, spx_swiglu_backward_rows)             */
} spx_layer_outputs;

/* Stage boundaries recorded into spx_layer_outputs.stage_events:
 * [0] start  [1] router GEMM done  [2] top-k done  [3] dispatch done
 * [4] expert GEMM1+SwiGLU done  [5] expert GEMM2 done  [6] shared GEMM1 done
 * [7] shared GEMM2 + combine done (end). */
#define SPX_STAGE_EVENTS 8

int spx_abi_version(void);
const char* spx_status_string(int status);

/* Columns of spx_layer_outputs.saved_gu for `dims` (chunk layout: per chunk
 * of the hidden width, its gate columns then its up columns). */
int spx_layer_saved_gu_cols(const spx_layer_dims* dims, int64_t* cols);
int spx_layer_saved_shared_gu(const spx_layer_dims* dims, int64_t* cols, int32_t* chunk);

/* Workspace bytes and packed weight sizes for `dims`. Host-only, no GPU work. */
int spx_layer_sizes(const spx_layer_dims* dims, size_t* workspace_bytes, spx_packed_sizes* packed);

/* BF16 -> BF16 softplus table (beta 1, threshold 20) for all 65536 inputs. */
int spx_softplus_table(uint16_t* table, void* stream);

/* Repack the reference state_dict into the kernel layouts (outputs sized by spx_layer_sizes).
 * expert_w1/expert_w2 may be NULL (with gate/up/down) to pack only the router
 * and shared weights. */
int spx_pack_weights(const spx_layer_dims* dims, const spx_reference_weights* src,
                     uint16_t* router_weight, uint16_t* expert_w1, uint16_t* expert_w2,
                     uint16_t* shared_w1, uint16_t* shared_w2, void* stream);

/* Quantise the expert masters for the MXFP8 lane (dims->mxfp8_lane = 1):
 * gate/up/down from the reference layouts into E4M3 copies with E8M0 scale
 * atoms (sizes from spx_layer_sizes).  Returns SPX_ERR_UNSUPPORTED when
 * inter_dim % 32 != 0. */
int spx_pack_weights_mxfp8(const spx_layer_dims* dims, const spx_reference_weights* src, uint8_t* expert_w1_mx,
                           uint8_t* expert_w1_mx_scales, uint8_t* expert_w2_mx, uint8_t* expert_w2_mx_scales,
                           void* stream);

/* MXFP8 quantisation of BF16 rows [rows, cols] along cols (cols % 32 == 0):
 * values[rows, cols] E4M3, scales[rows, cols / 32] E8M0 (RCEIL: byte =
 * clamp(ceil(log2(amax / 448)), -127, 127) + 127, multiplier 1 for byte 0). */
int spx_mxfp8_quantize_rows(const uint16_t* src, int64_t rows, int32_t cols, uint8_t* values, uint8_t* scales,
                            void* stream);

/* Workspace bytes of spx_mxfp8_mm_nt for the given shape. Host-only. */
size_t spx_mxfp8_mm_workspace(int64_t m, int64_t n, int64_t k);

/* out[m, n] = bf16(mx(left[m, k]) @ mx(right_rows[n, k]).T), FP32 accumulation
 * on the block-scaled tensor cores; K is zero-padded to a multiple of 128 as
 * in the reference.  BF16 inputs row-major, output row-major [m, n]. */
int spx_mxfp8_mm_nt(const uint16_t* left, const uint16_t* right_rows, int64_t m, int64_t n, int64_t k,
                    uint16_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* Scores, top-k ids and routing weights from given BF16 router logits [T, E]. */
int spx_route(const spx_layer_dims* dims, const uint16_t* logits, const uint16_t* softplus_table,
              const uint8_t* resident_mask, uint16_t* router_scores, int64_t* expert_ids,
              uint16_t* routing_weights, void* workspace, void* stream);

/* SurpriseRouter.forward (experts/router.py:40-56): router_scores [T, E] =
 * softplus(hidden @ W^T + b) in BF16 (the logits themselves for the legacy
 * identity transform).  Uses weights->router_weight (packed by
 * spx_pack_weights), ->router_bias and ->softplus_table; the workspace
 * (spx_router_sizes bytes, zero-filled once) holds the status word and the
 * K-padded rows when d_model % 64 != 0. */
int spx_router_sizes(const spx_layer_dims* dims, size_t* workspace_bytes);
int spx_router_forward(const spx_layer_dims* dims, const spx_packed_weights* weights,
                       const uint16_t* hidden, uint16_t* router_scores, void* workspace, void* stream);

/* Stable permutation of the T*k pairs by expert id, plus per-expert counts. */
int spx_dispatch(const spx_layer_dims* dims, const int64_t* expert_ids, int32_t* order,
                 int32_t* counts, void* workspace, void* stream);

/* One full layer forward: router GEMM, selection, dispatch, grouped expert
 * SwiGLU, shared SwiGLU and combine, routing statistics and auxiliary loss.
 * No host synchronisation. */
int spx_layer_forward(const spx_layer_dims* dims, const spx_packed_weights* weights,
                      const uint16_t* hidden, const spx_layer_outputs* outputs, void* workspace,
                      void* stream);

/* Router GEMM (or dims' injected logits), selection and dispatch of `hidden`
 * [T, d]: fills router_scores, expert_ids, routing_weights, the statistics,
 * dispatch_order, expert_counts and pair_rank (all required but the
 * statistics).  No expert or shared work. */
int spx_layer_route(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* hidden,
                    const spx_layer_outputs* outputs, void* workspace, void* stream);

/* out[i, :] = src[index[i] / index_div, :] for BF16 rows of d elements. */
int spx_gather_rows(const uint16_t* src, int64_t ld_src, const int32_t* index, int32_t index_div, int64_t rows,
                    int32_t d, uint16_t* out, int64_t ld_out, void* stream);

/* SwiGLU backward of rows (the autograd of nn/ffn.py:27-30 and of the
 * routed experts' silu(x W_g) * (x W_u), experts/bank.py:740-763, with the
 * routing weight applied to the upstream gradient).  gate_up [rows,
 * ld_gate_up] holds each row's pre-activations in chunks of `chunk` columns
 * ([gate chunk | up chunk] per chunk, inter / chunk chunks), d_hidden
 * [rows, ld_d_hidden] the gradient of the down projection's input before
 * the weight, weights[rows] BF16 routing weights (1 for unweighted rows).
 * Writes hidden [rows, inter] = bf16(bf16(bf16(silu(gate)) * up) * weight), d_gate_up
 * [rows, 2 * inter_pad] = [d gate | d up] (each half zero-padded to
 * inter_pad columns) and d_weights[order[r]] = sum over the row of
 * d_hidden * hidden (FP32).  Every intermediate is rounded to BF16.  Needs
 * chunk % 8 == 0, inter_pad % 8 == 0 and 16-byte aligned gate_up, d_hidden,
 * hidden and d_gate_up. */
int spx_swiglu_backward_rows(const uint16_t* gate_up, int64_t ld_gate_up, int32_t chunk, const uint16_t* d_hidden,
                             int64_t ld_d_hidden, const uint16_t* weights, const int32_t* order, int64_t rows,
                             int32_t inter, int32_t inter_pad, uint16_t* hidden, uint16_t* d_gate_up,
                             float* d_weights, void* stream);

/* Grouped SwiGLU experts of `rows` [R, d], row i through expert row_expert[i]
 * (0..num_experts-1 of `weights`): out_rows[i] = bf16(down(silu(gate x) *
 * up x)), unweighted, in input row order.  dims: tokens = R, top_k = 1,
 * num_experts = the local experts, shared_dim = 0. */
int spx_experts_forward(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* rows,
                        const int64_t* row_expert, uint16_t* out_rows, void* workspace, void* stream);
/* With out_rows NULL, spx_experts_forward leaves the outputs in dispatch
 * order inside the workspace: sorted_rows [R, d] and row_rank [R] (the
 * dispatch position of input row i), until the workspace's next use -- so a
 * caller can move them elsewhere (spx_rows_to_peers with index = row_rank)
 * in one pass. */
int spx_experts_sorted_rows(const spx_layer_dims* dims, void* workspace, const uint16_t** sorted_rows,
                            const int32_t** row_rank);
/* spx_experts_forward whose down-projection epilogue stores output row i
 * straight to row_out[i] (device array [R] of row pointers, each possibly in
 * a peer GPU's memory): the expert GEMM and the return exchange in one
 * kernel, the stores of a tile leaving as its epilogue runs. */
int spx_experts_forward_to(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* rows,
                           const int64_t* row_expert, uint16_t* const* row_out, void* workspace, void* stream);
/* spx_experts_forward_to whose gate/up GEMM reads input row i from
 * row_ptrs[i] (device array [R] of row pointers, each possibly in a peer
 * GPU's memory): the dispatch exchange folded into the GEMM's row gather.
 * BF16 experts only, d_model a multiple of 64 (SPX_ERR_UNSUPPORTED otherwise). */
int spx_experts_forward_rows(const spx_layer_dims* dims, const spx_packed_weights* weights,
                             const uint16_t* const* row_ptrs, const int64_t* row_expert, uint16_t* const* row_out,
                             void* workspace, void* stream);
/* Row pointers of the rows a rank receives, in its senders' memory: received
 * row i from sender g (recv_seg[g] <= i < recv_seg[g+1]) is g's pair at
 * dispatch position send_at[g] + i - recv_seg[g], whose token is
 * sender_order[g][pos] / top_k; row_ptrs[i] = sender_rows[g] + token * ld_rows.
 * All arrays are device arrays ([groups], [groups+1], [rows]). */
int spx_peer_row_pointers(const int32_t* const* sender_order, const int64_t* send_at, const int64_t* recv_seg,
                          int32_t groups, int32_t top_k, const uint16_t* const* sender_rows, int64_t ld_rows,
                          int64_t rows, const uint16_t** row_ptrs, void* stream);

/* Shared SwiGLU of `hidden` [T, d] into shared_out [T, d] (dims->shared_dim > 0). */
int spx_shared_forward(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* hidden,
                       uint16_t* shared_out, void* workspace, void* stream);

/* update[t] = bf16(shared[t] + sum_j bf16(expert_rows[pair_rank[t*k+j]] * w[t*k+j]))
 * in FP32, slots in order; pair_weights NULL = rows already weighted, shared
 * NULL = no shared path, a negative pair_rank = an empty slot. */
int spx_combine(const uint16_t* expert_rows, const int32_t* pair_rank, const uint16_t* pair_weights,
                const uint16_t* shared, int64_t tokens, int32_t d, int32_t top_k, uint16_t* update, void* stream);

/* Router calibration loss term and per-expert NLL attribution of one layer
 * (the reference's _attach_surprise_telemetry / _attribute_nll_to_experts,
 * modeling.py:1468-1534).  Inputs: the layer's router_scores [B, S, E],
 * expert_ids [B, S, k] and routing_weights [B, S, k], the next-token NLL
 * [B, S-1] (float) and its validity mask [B, S-1] (0/1 bytes).  Outputs
 * (any may be NULL): the mean smooth-L1 calibration loss over valid
 * positions (float scalar; NaN when none is valid), expert_attributed_nll [E]
 * and potentiation_utilization [E] (float).  Deterministic. */
size_t spx_calibration_workspace(int64_t batch, int64_t seq, int32_t num_experts);
int spx_surprise_calibration(const uint16_t* router_scores, const int64_t* expert_ids, const uint16_t* routing_weights,
                             const float* token_nll, const uint8_t* valid, int64_t batch, int64_t seq,
                             int32_t num_experts, int32_t top_k, float* calibration, float* attributed_nll,
                             float* utilization, void* workspace, size_t workspace_bytes, void* stream);

/* The channel half of a block: h_out = h + update, update = the layer
 * applied to channel_norm(h) (mESmaC/spalmer modeling.py:283-302 with
 * nn/norm.py:28-31 RMSNorm).  The RMSNorm is one pass writing the normalised
 * rows that every GEMM reads; the residual add runs in the combine.  Inputs
 * as spx_layer_forward plus the norm weight [d] (BF16) and eps; `hidden` is
 * the residual stream h; outputs as spx_layer_forward except that
 * outputs->update may be NULL (then only hidden_out = bf16(h + update) is
 * written) and injected logits are not accepted.  Same workspace. */
int spx_block_channel_forward(const spx_layer_dims* dims, const spx_packed_weights* weights,
                              const uint16_t* norm_weight, float eps, const uint16_t* hidden,
                              const spx_layer_outputs* outputs, uint16_t* hidden_out, void* workspace, void* stream);

/* Reconstruction error of each expert's low-precision copies
 * (MicroExpertBank.quantization_error with native_weight_reconstruction_error,
 * mESmaC/spalmer experts/bank.py:568-592 and experts/native.py:391-417): for
 * gate, up and down of expert e, W^T quantised row-wise along K (weight_format
 * 1 = MXFP8, 2 = NVFP4 under the matrix's own per-tensor scale) and
 * sum((W - bf16(deq))^2) / max(sum(W^2), 1e-12); expert_error[e] = the mean of
 * the three (float).  From the BF16 masters in src; dims gives E, d, I.
 * Compute it whenever the masters change and pass it as
 * spx_packed_weights.expert_quant_error. */
int spx_expert_quant_error(const spx_layer_dims* dims, const spx_reference_weights* src, int32_t weight_format,
                           float* expert_error, void* stream);

/* RMSNorm.forward (mESmaC/spalmer nn/norm.py:28-31) of BF16 rows: out[r] =
 * bf16(bf16(h[r] * bf16(rsqrt(mean(float(h[r])^2) + eps))) * weight), the
 * pass spx_block_channel_forward runs before the layer.  hidden [rows, d],
 * out [rows, ld_out] with columns d..ld_out zeroed (ld_out >= d); d and
 * ld_out multiples of 8, pointers 16-byte aligned, eps > 0.  The float sum
 * of squares runs in the device's own order. */
int spx_rmsnorm_rows(const uint16_t* hidden, const uint16_t* norm_weight, float eps, int64_t rows, int32_t d,
                     uint16_t* out, int32_t ld_out, void* stream);

/* ---- NVFP4 (experts/native.py:205-302, the ("nvfp4", "nvfp4") pair)
 * E2M1 values (two per byte, the even element in the low nibble), one UE4M3
 * scale per 16 elements along K, one FP32 per-tensor scale amax / (448 * 6)
 * per operand -- NVFP4Tensor.to_nvfp4(v, per_tensor_scale=...), restated.
 * spx_nvfp4_quantize_rows: _pack_nvfp4 of a BF16 matrix [rows, cols]:
 *   values [rows, kp/2] bytes, scales [rows, kp/16] bytes (kp = cols rounded
 *   up to 256, zero beyond cols), *amax = the matrix's largest |v| (float,
 *   device).
 * spx_nvfp4_mm_nt: native_nvfp4_linear's forward, out [m, n] =
 *   bf16(pts_l * pts_r * (deq(left) @ deq(right_rows)^T)) with FP32
 *   accumulation on tcgen05 kind::mxf4nvf4 MMAs (K = 64, block16 scales);
 *   workspace from spx_nvfp4_mm_workspace. */
int spx_nvfp4_quantize_rows(const uint16_t* src, int64_t rows, int32_t cols, uint8_t* values, uint8_t* scales,
                            float* amax, void* stream);
/* NVFP4 copies of the expert masters for a layer whose dims->mxfp8_lane == 2
 * (sizes: the *_mx fields of spx_layer_sizes): E2M1 gate|up chunks and down
 * rows with their scale atoms, each matrix under its own per-tensor scale,
 * and expert_amax [E][4] (gate, up, down, unused).  The activations get one
 * per-tensor scale per expert and forward (each expert's input is one call of
 * the reference's NVFP4 matmul). */
int spx_pack_weights_nvfp4(const spx_layer_dims* dims, const spx_reference_weights* src, uint8_t* expert_w1_nv,
                           uint8_t* expert_w1_nv_scales, uint8_t* expert_w2_nv, uint8_t* expert_w2_nv_scales,
                           float* expert_amax, void* stream);
size_t spx_nvfp4_mm_workspace(int64_t m, int64_t n, int64_t k);
int spx_nvfp4_mm_nt(const uint16_t* left, const uint16_t* right_rows, int64_t m, int64_t n, int64_t k,
                    uint16_t* out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- paged experts: the layer forward around a bounded device cache of expert weights
 * Reference: MicroExpertBank._execute_paged_grouped (experts/bank.py:821-899)
 * with the cache of offload.py / bank.py:241-365: routing over the full pool,
 * then the selected experts run page by page, each page's weights staged
 * into the cache first.  Three calls share one workspace (spx_layer_sizes of
 * `dims`) and run in order on `stream`:
 *   spx_layer_paged_begin    router, selection, dispatch (outputs as
 *                            spx_layer_forward; expert_counts required: the
 *                            host plans the pages from it), the MXFP8
 *                            quantisation of the hidden rows, shared GEMM1.
 *                            Expert weights are not read.
 *   spx_layer_paged_experts  the expert GEMMs of every pair whose expert e has
 *                            page_slot[e] >= 0 ([E] int32, device), reading
 *                            that expert's packed weights from slot
 *                            page_slot[e] of `cache` (expert_w1 / expert_w2 and
 *                            the MXFP8 copies laid out as spx_pack_weights
 *                            lays out cache_slots experts; expert_lane_mxfp8
 *                            as given to begin).  Call once per page; every
 *                            routed expert must be in exactly one page.
 *                            sm_limit > 0 caps the GEMMs' persistent grids
 *                            at that many SMs, leaving the others to a
 *                            concurrent spx_stage_expert_slots (0 = all).
 *   spx_layer_paged_finish   shared down projection and combine into
 *                            outputs->update (same outputs as begin).
 * The pages write the same rows an unpaged pass writes, so the update is
 * bit-identical to spx_layer_forward's. */
int spx_layer_paged_begin(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* hidden,
                          const spx_layer_outputs* outputs, void* workspace, void* stream);
int spx_layer_paged_experts(const spx_layer_dims* dims, const spx_packed_weights* cache, int32_t cache_slots,
                            const int32_t* page_slot, int32_t sm_limit, const uint16_t* hidden, void* workspace,
                            void* stream);
int spx_layer_paged_finish(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* hidden,
                           const spx_layer_outputs* outputs, void* workspace, void* stream);

/* Stage whole experts into cache slots (the copy half of _stage_expert_rows,
 * experts/bank.py:275-306): for each of the n (expert, slot) pairs (device
 * int32 [n][2]) and each of the `arrays` (<= 8) packed arrays,
 *   dst[a] + slot * bytes[a]  <-  src[a] + expert * bytes[a].
 * src, dst and bytes are host arrays of `arrays` entries; src[a] holds
 * num_experts experts and may be page-locked host memory (the GPU reads it
 * over the host link: one launch instead of one DMA copy per expert and
 * array); dst[a] (device) holds `slots` experts; bytes[a] % 16 == 0.
 * Pairs outside [0, num_experts) x [0, slots) are skipped.  `ctas` CTAs of
 * 512 threads (0 = 16) walk the blocks, so the copy occupies a few SMs. */
int spx_stage_expert_slots(const void* const* src, void* const* dst, const int64_t* bytes, int32_t arrays,
                           const int32_t* pairs, int32_t n, int32_t num_experts, int32_t slots, int32_t ctas,
                           void* stream);

/* ---- expert-parallel exchange over peer memory (NVLink / NVSwitch)
 * Each rank allocates its exchange buffers here (cudaMalloc) and publishes
 * the 64-byte CUDA IPC handle; peers open it as a device pointer of theirs.
 * spx_rows_to_peers stores rows straight into (peer) buffers: row i
 * (source row index[i] / index_div, or i when index is NULL) of segment g
 * (seg_offsets[g] <= i < seg_offsets[g+1]) goes to row dst_row_offsets[g] +
 * i - seg_offsets[g] of dst_ptrs[g] (row stride ld_dst).  seg_offsets
 * [groups+1], dst_ptrs [groups] and dst_row_offsets [groups] are device
 * arrays.  The kernel fences its stores at system scope; the caller orders
 * the peers' reads after it (a stream-ordered collective). */
int spx_ipc_buffer_alloc(size_t bytes, void** device_ptr, uint8_t* handle);
int spx_ipc_buffer_open(const uint8_t* handle, void** peer_ptr);
int spx_ipc_buffer_close(void* peer_ptr);
int spx_ipc_buffer_free(void* device_ptr);
int spx_rows_to_peers(const uint16_t* src, int64_t ld_src, const int32_t* index, int32_t index_div, int64_t rows,
                      int32_t d, const int64_t* seg_offsets, void* const* dst_ptrs, const int64_t* dst_row_offsets,
                      int64_t ld_dst, int32_t groups, void* stream);

/* ---- backward of the routed experts and the router scores
 * Reference: autograd through MicroExpertChannelMixer.forward
 * (experts/mixer.py:185-241: router.py:51-95, bank.py:705-779, 970-978,
 * losses.py:36-70), as training/engine.py:470 runs it.  Loss gradients in:
 * d_update (the update), d_aux (the auxiliary loss, optional) and d_scores
 * (router_scores, optional).  Out: the routed experts' part of dL/dx
 * (d_hidden_experts; the router's part is d_logits @ W_router and the shared
 * SwiGLU's is the caller's), dL/d logits, and the sorted-pair operands of the
 * expert weight gradients: with offsets from expert_counts,
 *   d gate_e | d up_e = x_sorted[e]^T @ dgu_sorted[e]   ([d, I] each, the up
 *                                                       half from column kI)
 *   d down_e          = h_sorted[e]^T @ du_sorted[e]    ([I, d]),
 * x_sorted[p] = hidden[token of p], du_sorted[p] = d_update[token of p] and
 * h_sorted[p] = bf16(h_p * w_p), pair p's forward hidden row times its
 * routing weight (the weight moved from dU to h: the same sum, its BF16
 * rounding on the narrow side).  x_sorted and du_sorted are both given or both
 * NULL; NULL needs the weight gradients below, whose kernels then gather
 * those rows by token themselves (no P x d copies are written).
 * BF16 experts only (SPX_ERR_UNSUPPORTED with an MXFP8 lane); d_model must be
 * a multiple of 64.  The dispatch is recomputed from expert_ids, so the
 * forward's workspace need not survive until the backward. */
typedef struct spx_layer_grads {
  const int64_t* expert_ids;        /* [T, k]  from the forward                  */
  const uint16_t* routing_weights;  /* [T, k]  from the forward (BF16)          */
  const uint16_t* router_scores;    /* [T, E]  from the forward (BF16)          */
  const uint16_t* gate_proj;        /* [E, d, I] reference layout (BF16)        */
  const uint16_t* up_proj;          /* [E, d, I]                                */
  const uint16_t* down_proj;        /* [E, I, d]                                */
  const uint16_t* d_update;         /* [T, d]  dL/d update                      */
  const uint16_t* d_scores;         /* [T, E]  dL/d router_scores | NULL        */
  const uint16_t* d_aux;            /* device BF16 scalar dL/d aux | NULL       */
  uint16_t* d_hidden_experts;       /* [T, d]  out                              */
  uint16_t* d_logits;               /* [T, E]  out                              */
  uint16_t* x_sorted;               /* [T*k, d]   out | NULL (with the wgrads)  */
  uint16_t* h_sorted;               /* [T*k, I]   out: bf16(hidden row * w)     */
  uint16_t* du_sorted;              /* [T*k, d]   out | NULL (with the wgrads)  */
  uint16_t* dgu_sorted;             /* [T*k, 2*kI] out, kI = round_up(I, 64)    */
  int32_t* expert_counts;           /* [E]     out                              */
  /* The routed experts' weight gradients (optional; NULL = not computed):
   * d gate | d up [E, d, I] = x_e^T [dg | du]_e and d down [E, I, d] =
   * h_e^T dy_e over each expert's sorted rows, FP32 accumulation, BF16 out
   * (tcgen05, both operands MN-major: from the sorted buffers above, or with
   * x_sorted = du_sorted = NULL gathered by token inside the kernels).  Needs
   * inter_dim % 8 == 0; all three or none. */
  uint16_t* d_gate_proj;
  uint16_t* d_up_proj;
  uint16_t* d_down_proj;
  /* The forward's saved_gu | NULL (GEMM1 recomputed).  With it, x_sorted
   * must hold the forward's saved_x: neither is written again. */
  const uint16_t* saved_gu;
  /* [T, E] the forward's router logits (spx_layer_outputs.router_logits) |
   * NULL (the router GEMM runs again; softplus scores only) */
  const uint16_t* router_logits;
  /* The workspace of the spx_layer_forward call these gradients belong to,
   * untouched since, with that call's expert_utilization ([E]): the
   * backward reads the forward's dispatch (sorted rows, tiles, ranks) from it
   * instead of dispatching again.  Both or neither (NULL: dispatch again from
   * expert_ids).  That forward must have left dispatch_order, expert_counts
   * and pair_rank NULL (they then live in its workspace). */
  const void* forward_workspace;
  const float* expert_utilization;
} spx_layer_grads;

int spx_layer_backward_sizes(const spx_layer_dims* dims, size_t* workspace_bytes);
int spx_layer_backward(const spx_layer_dims* dims, const spx_packed_weights* weights, const uint16_t* hidden,
                       const spx_layer_grads* grads, void* workspace, void* stream);

/* spx_dispatch without a workspace: same outputs, no device allocation by
 * anyone.  No counterpart in the reference; it exists for callers that cannot
 * allocate device memory (an FFI client holding only the buffers it was
 * handed, or code where cudaMalloc is forbidden or would synchronise, such as
 * global-mode stream capture).  Scratch is one file-scope device array of
 * about 6.2 MiB that every GPU loading libspx keeps until exit.  Limits:
 * tokens * top_k <= 1048576 and num_experts <= 1024, else
 * SPX_ERR_SCRATCH_LIMIT.  The first call on a device (with it current) looks
 * up the array's device address; make it before any stream capture.  Calls
 * share the array: calls that overlap on the GPU race, so serialise them.
 * `stream` must belong to the current device (else SPX_ERR_INVALID_ARG); the
 * looked-up address is kept for the life of the process (not refreshed
 * after cudaDeviceReset).  Expert ids outside [0, num_experts) are skipped,
 * their order slots are left unwritten, and the kernels record a non-zero
 * status word that spx_dispatch_static_status reads. */
int spx_dispatch_static(const spx_layer_dims* dims, const int64_t* expert_ids, int32_t* order,
                        int32_t* counts, void* stream);

/* Read (and clear when `clear` != 0) the status word that the kernels of the
 * last spx_dispatch_static call on the current device left in its scratch:
 * 0 = no error.  Synchronises `stream` (which must belong to the current
 * device); allocates nothing. */
int spx_dispatch_static_status(int* device_status, int clear, void* stream);

/* Read (and clear when `clear` != 0) the device status word of a workspace.
 * Synchronises `stream`.  *device_status == 0 means no kernel reported an error. */
int spx_workspace_status(void* workspace, int* device_status, int clear, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPX_H_ */
