/*
 * hs_ext.h — C ABI of libhs_ext.so, the B200 (sm_100a) kernels behind the
 * MTP speculative-decode MoE step of home-seek.
 *
 * Conventions (all entry points):
 *   - Pointers are raw DEVICE pointers, borrowed; outputs are caller-allocated.
 *   - Shapes are int64; `stream` is a cudaStream_t passed as void* (NULL = legacy
 *     default stream). Every launch is asynchronous on that stream.
 *   - The return value is an hs_status. Host-checkable errors (shape, alignment,
 *     workspace size, launch failure) are returned immediately. Data-dependent
 *     errors found on the device (expert id or token id out of range, a bounded
 *     wait that gave up) are OR-ed into the optional `dev_status` word (device
 *     int32, caller zeroes it) as HS_DEV_* bits; the host reads it when it syncs.
 *   - No entry point allocates device memory. Kernels that need scratch take a
 *     caller-provided `workspace`; its size comes from the matching
 *     *_workspace_size() query and it must be zero-filled once after allocation
 *     (the router's counter is left at zero by every call; the MoE call resets
 *     its own counters).
 *   - No exceptions, no global mutable state: concurrent calls on different
 *     streams are safe when they use different workspaces.
 *
 * The Python host layer (home_seek_b200/) binds this header with ctypes and
 * turns non-zero statuses into Python exceptions, which keeps the reference
 * engine's try/except fallback semantics.
 */
#ifndef HS_EXT_H
#define HS_EXT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HS_ABI_VERSION 2

typedef enum hs_status {
  HS_OK = 0,
  HS_ERR_BAD_SHAPE = 1,      /* a size or dimension the kernels do not support */
  HS_ERR_BAD_ARGUMENT = 2,   /* a NULL pointer where one is required, bad enum */
  HS_ERR_WORKSPACE = 3,      /* workspace smaller than *_workspace_size() */
  HS_ERR_ALIGN = 4,          /* pointer or stride not 16-byte aligned as required */
  HS_ERR_CUDA = 5,           /* a CUDA runtime/driver call failed */
  HS_ERR_UNSUPPORTED = 6,    /* device is not sm_100 or a driver entry point is missing */
  HS_ERR_NCCL = 7            /* an NCCL call failed (hs_ep_* over NCCL) */
} hs_status;

/* Bits OR-ed into the optional device status word. */
#define HS_DEV_BAD_EXPERT 0x1  /* an expert id outside [-1, E) was skipped */
#define HS_DEV_BAD_TOKEN 0x2   /* a token id outside [0, V) was skipped */
#define HS_DEV_TIMEOUT 0x4     /* a bounded device-side wait gave up */
#define HS_DEV_BAD_DRAFT 0x8   /* a draft id outside [0, V) */
#define HS_DEV_SMEM_ALIGN 0x10 /* dynamic shared memory not 1024-byte aligned; the MoE kernel did nothing */

int hs_abi_version(void);
/* Tracing builds (-DHS_TRACE, libhs_ext_trace.so): the device address of the  */
/* phase-stamp array (which = 0: [32 slots][5 kernels][296 CTAs][8 events]     */
/* u64 %globaltimer values) or of the layer-call counter (which = 1, u32);    */
/* NULL in the normal build.                                                   */
void* hs_trace_buffer(int which);
const char* hs_status_string(int status);
/* Last CUDA error code seen by the library on this thread (0 if none). */
int hs_last_cuda_error(void);

/* ------------------------------------------------------------------------ */
/* R1. Router: logits = bf16(h @ gate^T); logits = bf16(logits + bias);      */
/*     s = sqrt(softplus(f32(logits))); idx = stable top-k of s (ties to the  */
/*     lower expert id); w = s[idx] / max(sum, 1e-20) * routed_scaling.       */
/* Replaces home_seek/router.py:22-36 (compute_expert_affinity_with_bias)     */
/* and router.py:10-19 (compute_expert_affinity, bias == NULL), called from   */
/* inference_engine/engine.py:1025-1031 (_compute_routing_experts).           */
/* hidden [T][D] bf16, gate [E][D] bf16, bias [E] bf16 or NULL.               */
/* topk_idx [T][top_k] int64, topk_w [T][top_k] f32.                          */
/* logits_out [T][E] bf16 (post-bias) or NULL.                                */
/* Limits: D % 512 == 0, D <= 8192, E % 16 == 0, E <= 1024, top_k in [1, 16].  */
size_t hs_router_workspace_size(int64_t T, int64_t D, int64_t E);
int hs_router_topk(const void* hidden, const void* gate, const void* bias,
                   int64_t T, int64_t D, int64_t E, int64_t top_k,
                   float routed_scaling, int64_t* topk_idx, float* topk_w,
                   void* logits_out, void* workspace, size_t workspace_bytes,
                   void* stream);

/* R2. Hash routing for layers < num_hash_layers: idx = tid2eid[input_ids],   */
/*     w = 1/top_k. Replaces engine.py:1018-1023 (_compute_hash_experts).      */
/* input_ids [T] int64, tid2eid [V][top_k] int64 -> topk_idx [T][top_k] int64, */
/* topk_w [T][top_k] f32. Out-of-range ids give -1 and set HS_DEV_BAD_TOKEN.  */
int hs_hash_route(const int64_t* input_ids, int64_t T, const int64_t* tid2eid,
                  int64_t V, int64_t top_k, int64_t* topk_idx, float* topk_w,
                  int32_t* dev_status, void* stream);

/* ------------------------------------------------------------------------ */
/* R3/R5. Routed FP4 expert FFN with the FP8 shared expert fused in.          */
/*                                                                            */
/* Weight layout (what HBMExpertStore holds in HBM):                          */
/*   w13 [E][2][I][D/2]  u8  packed e2m1, low nibble = even column            */
/*   s13 [E][2][I/128][D/128][512] u8 ue8m0 scale-factor atoms (below)        */
/*   w2  [E][D][I/2]     u8  packed e2m1                                      */
/*   s2  [E][D/128][I/128][512]    u8 ue8m0 atoms                             */
/*   sh_w13 [2][I_sh][D] u8  e4m3 (w1 rows then w3 rows), or NULL            */
/*   sh_s13 [2][I_sh/128][D/128][512] u8 atoms of the 128x128 block scales    */
/*   sh_w2  [D][I_sh]    u8  e4m3                                             */
/*   sh_s2  [D/128][I_sh/128][512] u8 atoms                                   */
/* A scale-factor atom covers 128 rows x 128 columns (4 blocks of 32): byte   */
/* m0*16 + m1*4 + j holds the scale of row 32*m1 + m0, block j; the layout    */
/* tcgen05 scale-factor memory takes with one 32x128b copy. Row-major scales  */
/* s[R][C/32] convert with home_seek_b200/layout.py (scales_to_atoms).       */
/* Limits: D, I multiples of 512 in [512, 8192]; I_sh a multiple of 256 in    */
/* [256, 8192]; E <= 1024; w13/w2 32-byte aligned, other pointers 16-byte.    */
/* ------------------------------------------------------------------------ */
typedef struct hs_moe_weights {
  const void* w13;
  const void* s13;
  const void* w2;
  const void* s2;
  const void* sh_w13;
  const void* sh_s13;
  const void* sh_w2;
  const void* sh_s2;
  int64_t E;
  int64_t D;
  int64_t I;
  int64_t I_sh;
} hs_moe_weights;

/* Opaque per-layer descriptor (TMA tensor maps over the weights), encoded    */
/* once on the host by hs_moe_make_desc and passed by pointer to every call.  */
#define HS_MOE_DESC_BYTES 1024
int hs_moe_make_desc(const hs_moe_weights* weights, void* desc_out, size_t desc_bytes);

/* Duplicate (token, expert) pairs in one top-k row: */
#define HS_DUP_LAST 0 /* keep the last occurrence's weight (fused_moe.py:526-539) */
#define HS_DUP_SUM 1  /* sum the weights (engine.py:1388-1393, the T=1 path)     */

size_t hs_moe_workspace_size(int64_t T, int64_t top_k, int64_t D, int64_t I,
                             int64_t I_sh);

/* out[t] = bf16( bf16(sum_e w_te * FFN_e(h_t)) + bf16(FFN_shared(h_t)) )      */
/* with FFN(h) = bf16(bf16(clamp(g)*sigmoid(g)*clamp(u)) ...) exactly as       */
/* FusedMoEFFN._forward_legacy (fused_moe.py:458-551) plus                     */
/* SharedExpertFFN.forward / fused_expert_ffn_pt (fused_moe.py:383-392,        */
/* 573-598) and the bf16 add at engine.py:1530-1536.                           */
/* Replaces FusedMoEFFN.forward (fused_moe.py:447-456) and                     */
/* FusedMoEFFN.forward_m1_fp4 (fused_moe.py:553-563).                          */
/* hidden [T][D] bf16; topk_idx [T][top_k] int64 (-1 = skip); topk_w [T][top_k]*/
/* f32; out [T][D] bf16. out_f32 [T][D] f32 (optional, may be NULL) receives   */
/* the routed sum before rounding (used by the expert-parallel combine).       */
/* use_shared = 0 skips the shared expert even if the descriptor has one.      */
int hs_moe_ffn_fp4(const void* desc, const void* hidden, const int64_t* topk_idx,
                   const float* topk_w, int64_t T, int64_t top_k, int use_shared,
                   int dup_mode, void* out, float* out_f32, void* workspace,
                   size_t workspace_bytes, int32_t* dev_status, void* stream);

/* hs_moe_ffn_fp4_noalloc: hs_moe_ffn_fp4 without the workspace argument.     */
/* No counterpart in the reference. It is for callers that cannot allocate    */
/* device memory at the moment they call: plugin hosts whose enqueue path     */
/* forbids allocation, and latency-critical loops in which cudaMalloc or      */
/* cudaFree would synchronise the device. The scratch is                      */
/* a fixed array of HS_MOE_NOALLOC_BYTES inside the library; every GPU that   */
/* loads the library holds it until the process exits. A call whose          */
/* hs_moe_workspace_size(T, top_k, D, I, I_sh) exceeds it returns             */
/* HS_ERR_WORKSPACE without launching (on a 148-SM B200 at D = 4096,         */
/* I = I_sh = 2048, top_k = 6 --- the size grows with the SM count ---       */
/* that allows T <= 16 tokens). The first call on a device looks up the       */
/* array's device address (cudaGetSymbolAddress): make that first call        */
/* before any stream capture. The address is kept for the life of the        */
/* process: after cudaDeviceReset (or any teardown of the device's primary    */
/* context) it is stale, so do not call this entry point on that device again */
/* in the same process. All calls share the one array, so calls that          */
/* overlap on the GPU (two streams, two host threads) race; the kernels clear */
/* the counters they need at the start of every call.                         */
#define HS_MOE_NOALLOC_BYTES (16u << 20)
int hs_moe_ffn_fp4_noalloc(const void* desc, const void* hidden, const int64_t* topk_idx,
                           const float* topk_w, int64_t T, int64_t top_k, int use_shared,
                           int dup_mode, void* out, float* out_f32, int32_t* dev_status,
                           void* stream);

/* ------------------------------------------------------------------------ */
/* R10. Permute / unpermute, with the semantics of the reference's test       */
/* oracles tests/_reference.py:93-121 (expand_to_fused) and                   */
/* tests/_reference.py:52-90 (reduce_fused). Positions are expert-major       */
/* (ascending expert id, then ascending token), deterministic.                */
/* hs_moe_permute: topk_idx [T][k] -> token_topk_to_pos [T][k] int32 (-1 for  */
/*   invalid), pos_to_expert [T*k] int32 (-1 past the end), expert_count [E]   */
/*   int32, num_pos (device int32), and x_expanded [T*k][D] bf16 (may be NULL) */
/*   gathered from x [T][D] bf16.                                              */
/* hs_moe_unpermute: out[t] = cast(sum_k w[t][k] * x[pos[t][k]]) in f32, in    */
/*   k order, over valid positions; weights may be NULL (= 1).                 */
/* ------------------------------------------------------------------------ */
size_t hs_moe_permute_workspace_size(int64_t T, int64_t top_k, int64_t E);
int hs_moe_permute(const int64_t* topk_idx, int64_t T, int64_t top_k, int64_t E,
                   const void* x, int64_t D, int32_t* token_topk_to_pos,
                   int32_t* pos_to_expert, int32_t* expert_count, int32_t* num_pos,
                   void* x_expanded, void* workspace, size_t workspace_bytes,
                   int32_t* dev_status, void* stream);
int hs_moe_unpermute(const void* x_expanded, int64_t num_expanded, int64_t D,
                     const int32_t* token_topk_to_pos, const float* topk_w,
                     int64_t T, int64_t top_k, void* out_bf16, void* stream);

/* ------------------------------------------------------------------------ */
/* R6. Acceptance.                                                            */
/* hs_accept_greedy: logits [B][T][V] bf16 (row stride V); draft_ids [B][T-1] */
/*   int64. For each row b: n_accept = number of leading positions i < T-1    */
/*   with argmax(logits[b][i]) == draft_ids[b][i]; next_token =               */
/*   argmax(logits[b][n_accept]). argmax takes the first maximal index and   */
/*   treats NaN as maximal (torch.argmax). Replaces the loop at               */
/*   engine.py:2485-2497 and the t=0 bonus at engine.py:2908-2913.            */
/*   argmax_out [B][T] int64 may be NULL.                                     */
/* hs_accept_rejection: standard speculative sampling (Leviathan et al. 2023) */
/*   with p = softmax(target/t), q = softmax(draft/t) (f32, evaluated as      */
/*   2^((x - max) * log2(e) / t) with the hardware ex2): accept draft i       */
/*   iff u[b][i] < p_i(d_i) / q_i(d_i); at the first rejection i sample from  */
/*   normalise(max(0, p_i - q_i)), else (all accepted) from p_M, by inverse   */
/*   CDF in ascending token order with u[b][M]. target [B][M+1][V],           */
/*   draft [B][draft_rows][V] (draft_rows >= M), draft_ids [B][M],            */
/*   uniform [B][M+1] f32. t <= 0 falls back to greedy.                       */
/*   Outputs n_accept [B] int32 and next_token [B] int64.                     */
/* Limits: V >= 64, V*2 % 16 == 0 (rows 16-byte aligned).                     */
/* ------------------------------------------------------------------------ */
int hs_accept_greedy(const void* logits, int64_t B, int64_t T, int64_t V,
                     const int64_t* draft_ids, int32_t* n_accept,
                     int64_t* next_token, int64_t* argmax_out,
                     int32_t* dev_status, void* stream);
int hs_accept_rejection(const void* target_logits, const void* draft_logits,
                        int64_t B, int64_t M, int64_t draft_rows, int64_t V,
                        const int64_t* draft_ids, const float* uniform,
                        float temperature, int32_t* n_accept,
                        int64_t* next_token, int32_t* dev_status, void* stream);

/* ------------------------------------------------------------------------ */
/* lm_head GEMV with the greedy decision fused in.                            */
/* Replaces `logits = h_3d @ lm_head.t()` + `argmax` of the MTP draft          */
/* (inference_engine/engine.py:2327-2333), of the fused verify with its greedy */
/* loop (engine.py:2482-2497) and of the main decode step                     */
/* (engine.py:2846-2853). x [T][D] bf16 (rows after the final norm), head     */
/* [V][D] bf16. logit[t][v] = bf16(sum_k x[t][k] * head[v][k]) with f32        */
/* accumulation; the logits stay on chip unless logits_out [T][V] bf16 is     */
/* given. argmax_out [T] int64 (may be NULL) = first index of the maximal      */
/* logit of row t, NaN maximal (torch.argmax). With draft_ids [T-1] (T > 1;   */
/* may be NULL): n_accept = number of leading positions i < T-1 with          */
/* argmax[i] == draft_ids[i], next_token = argmax[n_accept]; without draft    */
/* ids n_accept = 0 and next_token = argmax[0]. n_accept [1] int32 and        */
/* next_token [1] int64 may be NULL. A draft id outside [0, V) stops the      */
/* acceptance there and sets HS_DEV_BAD_DRAFT. The workspace (size from        */
/* hs_lm_head_workspace_size, zero-filled once) holds one key per CTA and     */
/* token and a counter the call leaves at zero.                               */
/* Limits: 1 <= T <= 16, D a multiple of 64 (<= 65536), V <= 2^30; x and head */
/* 16-byte aligned; logits_out needs V % 8 == 0.                               */
/* ------------------------------------------------------------------------ */
size_t hs_lm_head_workspace_size(int64_t T);
int hs_lm_head_argmax(const void* x, const void* head, int64_t T, int64_t D,
                      int64_t V, const int64_t* draft_ids, int64_t* argmax_out,
                      int32_t* n_accept, int64_t* next_token, void* logits_out,
                      void* workspace, size_t workspace_bytes,
                      int32_t* dev_status, void* stream);

/* ------------------------------------------------------------------------ */
/* RMSNorm and residual add + RMSNorm (the layer loop around the MoE FFN).    */
/* hs_rms_norm replaces home_seek/utils.py:6-9 (rms_norm; called before every */
/*   FFN at inference_engine/engine.py:2679 and before the logits at          */
/*   engine.py:2482): out = bf16(f32(w) * (f32(x) * 1/sqrt(mean(x^2) + eps))). */
/* hs_add_rms_norm fuses the residual add that closes a layer                 */
/*   (engine.py:2685, h = h + ffn_out) with the norm that opens the next:     */
/*   h_out = bf16(h + y), x_out = rms_norm(h_out, w). h_out may alias h.       */
/*   w and x_out both NULL: the residual add alone (h_out = bf16(h + y)).     */
/* x, h, y, w, out: bf16, rows of D; T rows. Limits: D % 8 == 0, D <= 8192,    */
/* 16-byte aligned pointers. The sum of squares runs in a fixed order         */
/* (deterministic; it may differ from torch's by an ulp of the variance).     */
/* ------------------------------------------------------------------------ */
int hs_rms_norm(const void* x, const void* w, float eps, int64_t T, int64_t D,
                void* out, void* stream);
int hs_add_rms_norm(const void* h, const void* y, const void* w, float eps,
                    int64_t T, int64_t D, void* h_out, void* x_out,
                    void* stream);

/* ------------------------------------------------------------------------ */
/* Expert parallelism: partial sums and their combine.                        */
/* The reference splits the experts of a layer across GPUs, runs every GPU    */
/* on all tokens and adds the outputs (engine.py:1575-1709 _forward_ffn_ep,   */
/* parallel.py:203-290 _EPWorker). Here each rank runs                        */
/* hs_moe_ffn_fp4_partials on its experts (ids outside them set to -1) and    */
/* its slice of the shared expert's intermediate dimension, writing the       */
/* UN-ROUNDED f32 sums routed_f32 [T][D] and shared_f32 [T][D]; the caller    */
/* sums those over ranks (one NCCL all-reduce) and hs_moe_combine rounds them */
/* exactly as the single-GPU call does: out = bf16(bf16(routed) +             */
/* bf16(shared)). hs_moe_combine_add_rms_norm fuses the combine with the      */
/* layer's residual add and the next norm (as hs_add_rms_norm).               */
/* shared_f32 is required when use_shared (and the descriptor has a shared    */
/* expert); pointers 16-byte aligned.                                         */
/* ------------------------------------------------------------------------ */
int hs_moe_ffn_fp4_partials(const void* desc, const void* hidden,
                            const int64_t* topk_idx, const float* topk_w,
                            int64_t T, int64_t top_k, int use_shared,
                            int dup_mode, float* routed_f32, float* shared_f32,
                            void* workspace, size_t workspace_bytes,
                            int32_t* dev_status, void* stream);
/* ------------------------------------------------------------------------ */
/* Routing folded into the MoE call (decode sizes).                          */
/* One call = hs_router_topk + hs_moe_ffn_fp4 (or its partials form) for     */
/* T <= 8 tokens: the router (router.py:22-36, same arithmetic and           */
/* selections as hs_router_topk) runs in one thread-block cluster that also  */
/* builds the FFN's plan, so the layer is three launches instead of five.    */
/* hidden [T][D] bf16 (normed rows), gate [num_experts][D] bf16, bias         */
/* [num_experts] bf16 or NULL; topk_idx [T][top_k] int64 (global ids) and    */
/* topk_w [T][top_k] f32 receive the routing. The descriptor's store holds    */
/* routed experts [expert_offset, expert_offset + E) (expert parallelism;     */
/* 0 and num_experts for a full store); selections outside it are skipped.    */
/* Limits: T <= 8, 16 <= num_experts <= 256 (a multiple of 16), D <= 4096;   */
/* otherwise HS_ERR_UNSUPPORTED (use hs_router_topk + hs_moe_ffn_fp4). The    */
/* workspace is hs_moe_workspace_size(T, top_k, D, I, I_sh).                  */
/* ------------------------------------------------------------------------ */
int hs_moe_route_ffn_fp4(const void* desc, const void* hidden,
                         const void* gate, const void* bias,
                         int64_t num_experts, int64_t expert_offset,
                         int64_t T, int64_t top_k, float routed_scaling,
                         int use_shared, int dup_mode, int64_t* topk_idx,
                         float* topk_w, void* out, float* out_f32,
                         void* workspace, size_t workspace_bytes,
                         int32_t* dev_status, void* stream);
int hs_moe_route_ffn_fp4_partials(const void* desc, const void* hidden,
                                  const void* gate, const void* bias,
                                  int64_t num_experts, int64_t expert_offset,
                                  int64_t T, int64_t top_k,
                                  float routed_scaling, int use_shared,
                                  int dup_mode, int64_t* topk_idx,
                                  float* topk_w, float* routed_f32,
                                  float* shared_f32, void* workspace,
                                  size_t workspace_bytes, int32_t* dev_status,
                                  void* stream);
/* ------------------------------------------------------------------------ */
/* The MoE half of a decode layer in one call (T <= 8).                       */
/* h_out = h + MoE(rms_norm(h, norm_w)): the norm that opens the FFN block    */
/* (engine.py:2679, utils.py:6-9), the routing, the routed FP4 experts with   */
/* the FP8 shared expert, and the residual add that closes the layer          */
/* (engine.py:2685), in three launches: the norm runs inside the routing      */
/* cluster (same summation order as hs_rms_norm, so the rows are identical)   */
/* and the add inside the down phase's epilogue. Routing is the router        */
/* (gate, bias, routed_scaling; as hs_moe_route_ffn_fp4) or, when tid2eid is  */
/* not NULL, hash routing by input_ids (as hs_hash_route: weights 1/top_k,    */
/* gate and bias ignored). x_out [T][D] receives the normed rows when not     */
/* NULL. h_out may alias h. The partials form writes the UN-ROUNDED f32 sums  */
/* of this rank's experts instead (expert parallelism); the caller adds them  */
/* over ranks and calls hs_moe_combine_add_rms_norm with w = x_out = NULL for */
/* h_out = h + combine. No reference entry point has this shape: it replaces  */
/* the FFN block of _forward_layer (engine.py:2679-2685) as one operator.     */
/* Limits and workspace as hs_moe_route_ffn_fp4.                              */
/* ------------------------------------------------------------------------ */
int hs_moe_layer_fp4(const void* desc, const void* h, const void* norm_w,
                     float eps, const void* gate, const void* bias,
                     const int64_t* input_ids, const int64_t* tid2eid,
                     int64_t vocab, int64_t num_experts, int64_t expert_offset,
                     int64_t T, int64_t top_k, float routed_scaling,
                     int use_shared, int dup_mode, int64_t* topk_idx,
                     float* topk_w, void* x_out, void* h_out, void* workspace,
                     size_t workspace_bytes, int32_t* dev_status, void* stream);
int hs_moe_layer_fp4_partials(const void* desc, const void* h,
                              const void* norm_w, float eps, const void* gate,
                              const void* bias, const int64_t* input_ids,
                              const int64_t* tid2eid, int64_t vocab,
                              int64_t num_experts, int64_t expert_offset,
                              int64_t T, int64_t top_k, float routed_scaling,
                              int use_shared, int dup_mode, int64_t* topk_idx,
                              float* topk_w, void* x_out, float* routed_f32,
                              float* shared_f32, void* workspace,
                              size_t workspace_bytes, int32_t* dev_status,
                              void* stream);
/* ------------------------------------------------------------------------ */
/* Expert parallelism over NVLink peer memory (decode sizes, T <= 8).         */
/* The reference's EP adds the GPUs' outputs on GPU 0 (engine.py:1575-1709,  */
/* parallel.py:203-290); hs_moe_layer_fp4_partials + an NCCL all-reduce is    */
/* this library's collective form of it. hs_moe_layer_fp4_ep fuses the        */
/* exchange into the layer call instead: the down phase stores each rank's    */
/* f32 routed/shared rows straight into every rank's receive buffer over      */
/* NVLink (plain peer stores, no multicast; an entry is empty until stored,   */
/* so the entries are their own arrival flags); a combine kernel waits        */
/* (bounded) for this call's entries of all ranks, sums them in rank order    */
/* (so every rank holds the same h), applies bf16(bf16(routed) +              */
/* bf16(shared)) and the residual add, and empties the entries again. Setup,  */
/* once per process and rank: hs_ep_buffer_alloc a buffer of                  */
/* hs_ep_buffer_bytes(world, D) (zero-filled), exchange its handle from       */
/* hs_ipc_get_handle with the other ranks, hs_ipc_open_handle theirs, and     */
/* fill hs_ep_peers (recv[q] = rank q's buffer as mapped here, recv[rank] =   */
/* the local one). Every rank must make the same sequence of calls. Limits:   */
/* world <= HS_EP_MAX_RANKS, T <= 8, D <= 8192; the down phase must run on     */
/* clusters (D = 4096 on a B200), else HS_ERR_UNSUPPORTED.                     */
/* Failure: the combine waits at most wait_limit_ns (0 = two seconds) for a    */
/* peer's entries. When a wait runs out it sets HS_DEV_TIMEOUT, marks the      */
/* local buffer poisoned and leaves the call counter where it was, so rows a  */
/* late peer stores afterwards are never read as a later call's data. Every   */
/* later call on a poisoned buffer stores nothing to the peers and its        */
/* combine reports HS_DEV_TIMEOUT at once without waiting or writing h_out;   */
/* the group must free and re-create its buffers (hs_ep_buffer_alloc) before */
/* exchanging again.                                                          */
/* ------------------------------------------------------------------------ */
#define HS_EP_MAX_RANKS 8
#define HS_IPC_HANDLE_BYTES 64
typedef struct hs_ep_peers {
  int32_t rank, world;
  void* recv[HS_EP_MAX_RANKS];
  int64_t wait_limit_ns;  /* bound of the combine's wait for peers; 0 = 2 s */
} hs_ep_peers;
size_t hs_ep_buffer_bytes(int64_t world, int64_t D);
int hs_ep_buffer_alloc(size_t bytes, void** ptr);
int hs_ep_buffer_free(void* ptr);
int hs_ipc_get_handle(const void* ptr, void* handle, size_t handle_bytes);
int hs_ipc_open_handle(const void* handle, void** ptr);
int hs_ipc_close_handle(void* ptr);
int hs_moe_layer_fp4_ep(const void* desc, const void* h, const void* norm_w,
                        float eps, const void* gate, const void* bias,
                        const int64_t* input_ids, const int64_t* tid2eid,
                        int64_t vocab, int64_t num_experts,
                        int64_t expert_offset, int64_t T, int64_t top_k,
                        float routed_scaling, int use_shared, int dup_mode,
                        int64_t* topk_idx, float* topk_w, void* x_out,
                        const hs_ep_peers* peers, void* h_out, void* workspace,
                        size_t workspace_bytes, int32_t* dev_status,
                        void* stream);
/* hs_moe_layer_fp4_ep_chained: hs_moe_layer_fp4_ep for a stack of layers    */
/* with the exchange of one call completed at the start of the next. The      */
/* rows h are read and written in place: with prev_pending set, the route     */
/* kernel first adds the previous chained call's MoE output (prev_use_shared  */
/* its use_shared) to h exactly as hs_moe_layer_fp4_ep's combine does, then   */
/* routes on the result; this call's own output stays pending in the receive  */
/* buffers. hs_ep_combine_pending(peers, h, T, D, use_shared) completes the   */
/* last pending call (its combine kernel alone, h_out = h). Consecutive       */
/* chained calls take the same h, T and D, and every rank makes the same      */
/* sequence of calls; failure behaves as in hs_moe_layer_fp4_ep.              */
int hs_moe_layer_fp4_ep_chained(const void* desc, void* h, const void* norm_w,
                                float eps, const void* gate, const void* bias,
                                const int64_t* input_ids,
                                const int64_t* tid2eid, int64_t vocab,
                                int64_t num_experts, int64_t expert_offset,
                                int64_t T, int64_t top_k, float routed_scaling,
                                int use_shared, int dup_mode, int64_t* topk_idx,
                                float* topk_w, void* x_out,
                                const hs_ep_peers* peers, int prev_pending,
                                int prev_use_shared, void* workspace,
                                size_t workspace_bytes, int32_t* dev_status,
                                void* stream);
int hs_ep_combine_pending(const hs_ep_peers* peers, void* h, int64_t T,
                          int64_t D, int use_shared, int32_t* dev_status,
                          void* stream);
/* hs_lm_head_argmax_ep: hs_lm_head_argmax with the vocabulary split over the */
/* same group (no counterpart in the reference, whose lm_head runs on one      */
/* GPU). head_rows points at rows [row0, row0 + rows) of the [V][D] head: this */
/* rank streams only those, finds each token's best (bf16 logit, first index) */
/* over them (global indices), stores those T keys into every rank's exchange */
/* buffer and waits (bounded, as the MoE combine: HS_DEV_TIMEOUT and a poison */
/* word on expiry) for every rank's, so argmax_out, n_accept and next_token   */
/* are those of hs_lm_head_argmax on the whole head, on every rank. Every     */
/* rank makes the same calls; the rows of the ranks tile [0, V). No logits    */
/* output; T <= 16, D <= 8192.                                                 */
int hs_lm_head_argmax_ep(const void* x, const void* head_rows, int64_t T,
                         int64_t D, int64_t V, int64_t row0, int64_t rows,
                         const int64_t* draft_ids, int64_t* argmax_out,
                         int32_t* n_accept, int64_t* next_token,
                         const hs_ep_peers* peers, void* workspace,
                         size_t workspace_bytes, int32_t* dev_status,
                         void* stream);
int hs_moe_combine(const float* routed_f32, const float* shared_f32,
                   int use_shared, int64_t T, int64_t D, void* out,
                   void* stream);
int hs_moe_combine_add_rms_norm(const float* routed_f32,
                                const float* shared_f32, int use_shared,
                                const void* h, const void* w, float eps,
                                int64_t T, int64_t D, void* h_out, void* x_out,
                                void* stream);

/* ------------------------------------------------------------------------ */
/* Expert parallelism with the tokens sharded over the ranks (prefill), one  */
/* call over NCCL. Replaces the reference's _forward_ffn_ep                  */
/* (inference_engine/engine.py:1575-1709: every token on every GPU, the GPUs' */
/* bf16 expert outputs added) and the dispatch/combine of                     */
/* inference_engine/parallel.py:189-384. Rank r owns a shard of the tokens,  */
/* its routing (global expert ids), and a store with the routed experts       */
/* [r E_l, (r+1) E_l) (E_l = the descriptor's E) and the whole shared expert. */
/* hs_ep_dispatch_combine, on the caller's stream:                            */
/*   - sends each token's row once to every other rank holding one of its     */
/*     experts, with its ids localised there and its weights (NCCL send/recv, */
/*     after a count exchange read on the host: the call's one sync);         */
/*   - runs hs_moe_ffn_fp4_partials on the own tokens (own experts + shared)  */
/*     and on the received rows (routed only);                                */
/*   - returns the received rows' f32 sums, adds every token's terms in rank  */
/*     order (the own term at this rank's place) and writes                   */
/*     out = bf16(bf16(routed) + bf16(shared)) [T][D].                        */
/* Every rank of the communicator calls it with the same T_max (>= every     */
/* rank's T), top_k, use_shared and dup_mode and a workspace of at least      */
/* hs_ep_dispatch_combine_workspace_size(T_max, top_k, D, I, I_sh, world)     */
/* bytes (zero-filled once). A rank whose own arguments are bad (T > T_max,   */
/* NULL or unaligned pointers) takes part with no tokens and returns the      */
/* error afterwards, so its peers' calls complete. T may be 0. With world 1  */
/* the call makes no NCCL call and no host synchronisation. NCCL is loaded at */
/* run time (libnccl.so.2); without it these return HS_ERR_UNSUPPORTED.       */
/* T, T_max <= 65535; world <= HS_EP_MAX_RANKS.                                */
/* hs_ep_nccl_unique_id: on one rank; the caller hands the                    */
/* HS_NCCL_UNIQUE_ID_BYTES to the others. hs_ep_nccl_comm_init: on every rank */
/* with the current CUDA device set.                                          */
/* hs_ep_dispatch_plan: the call's first step alone (for tests and callers   */
/* with their own transport): counts[world] (rows to each rank; 0 for this   */
/* rank), pos[T][world] (the token's place in each rank's list, or -1),      */
/* own_ids[T][top_k] (this rank's ids localised, others -1; may be NULL).     */
/* ------------------------------------------------------------------------ */
#define HS_NCCL_UNIQUE_ID_BYTES 128
int hs_ep_nccl_unique_id(void* id_out);
int hs_ep_nccl_comm_init(const void* id, int32_t world, int32_t rank, void** comm);
int hs_ep_nccl_comm_destroy(void* comm);
int hs_ep_dispatch_plan(const int64_t* topk_idx, int64_t T, int64_t top_k,
                        int64_t experts_per_rank, int32_t world, int32_t rank,
                        int32_t* counts, int32_t* pos, int64_t* own_ids,
                        void* stream);
size_t hs_ep_dispatch_combine_workspace_size(int64_t T_max, int64_t top_k,
                                             int64_t D, int64_t I, int64_t I_sh,
                                             int32_t world);
int hs_ep_dispatch_combine(void* comm, const void* desc, const void* hidden,
                           const int64_t* topk_idx, const float* topk_w,
                           int64_t T, int64_t T_max, int64_t top_k,
                           int use_shared, int dup_mode, void* out,
                           void* workspace, size_t workspace_bytes,
                           int32_t* dev_status, void* stream);

/* ------------------------------------------------------------------------ */
/* Verify-state snapshot / restore on the device.                             */
/* Replaces the state handling of _mtp_verify_batched                         */
/* (inference_engine/engine.py:2443-2459, 2500-2538): the reference clones    */
/* every layer's KV latent cache, compressed KV and compressor state before   */
/* the fused verify forward and, unless every position was accepted, trims    */
/* the KV caches to old length + n_accept and puts the rest back. Here each   */
/* state is a region of a table in DEVICE memory (built once by the caller):  */
/*   append region (length != NULL): a device entry count. Snapshot records   */
/*     it in saved_length; commit sets *length = saved_length + n_accept when */
/*     keep_accepted (KV caches, the position), else saved_length.            */
/*   copy region (length == NULL): `bytes` at `live` (16-byte aligned, bytes  */
/*     a multiple of 16) saved into `shadow` (same size) by the snapshot and  */
/*     copied back by the commit (compressor states, compressed KV).          */
/* The commit does nothing when *n_accept >= t_total (all accepted), as the   */
/* reference. n_accept is device memory (e.g. hs_lm_head_argmax's output):    */
/* no host synchronisation. max_bytes = the largest copy region's size (it    */
/* sets the grid). One launch per call over all regions; n <= 65535.         */
/* ------------------------------------------------------------------------ */
typedef struct hs_state_region {
  void* live;
  void* shadow;
  int64_t bytes;
  int64_t* length;
  int64_t saved_length;
  int32_t keep_accepted;
  int32_t reserved;
} hs_state_region;
int hs_verify_state_snapshot(hs_state_region* regions, int64_t n,
                             int64_t max_bytes, void* stream);
int hs_verify_state_commit(hs_state_region* regions, int64_t n,
                           int64_t max_bytes, const int32_t* n_accept,
                           int32_t t_total, void* stream);

/* ------------------------------------------------------------------------ */
/* Synthetic weight fill (device-side, counter-based hash; no allocation).    */
/* Fills n bytes at dst with lo + (hash(seed, i) % (hi - lo + 1)). Used to    */
/* build random-init expert stores of the full model shape in seconds.        */
/* No counterpart in the reference (its weights come from safetensors).       */
/* ------------------------------------------------------------------------ */
int hs_fill_bytes(void* dst, int64_t n, uint64_t seed, int32_t lo, int32_t hi,
                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HS_EXT_H */
