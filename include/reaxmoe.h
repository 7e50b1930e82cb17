/*
 * reaxmoe.h -- C ABI of the B200 (sm_100a) NVFP4 prefill MoE layer.
 *
 * One entry point per stage of the reference's MoE operator, plus the whole layer. All pointers are device
 * pointers unless stated; every call is asynchronous on the given CUDA stream (passed as void*, i.e. a
 * cudaStream_t; NULL = the legacy default stream), allocates nothing, performs no host synchronisation and
 * returns an int status: 0 = ok, > 0 = one of the REAXMOE_ERR_* codes below. The text of the last error of
 * the calling thread is available from reaxmoe_last_error().
 *
 * Reference interfaces replaced (paths are within the reference project):
 *   - vLLM run_cutlass_moe_fp4(output, a, a1_gscale, w1_fp4, w1_blockscale, w1_alphas, a2_gscale, w2_fp4,
 *     w2_blockscale, w2_alphas, topk_weights, topk_ids, activation, workspace13, workspace2, m, n, k, e,
 *     ...), as patched by champions/uid240/opt/blink/blink_moe.py:434-567 (stock body:
 *     vllm/model_executor/layers/fused_moe/experts/cutlass_moe.py:481-664)      -> reaxmoe_forward
 *   - Gemma-4 routing function (vllm/model_executor/models/gemma4.py:95-203, called from
 *     gemma4.py:332-345)                                                          -> reaxmoe_route
 *   - Gemma4Router.forward (gemma4.py:251-298; champion router GEMM blink_rgemm.cu:44-56) + the routing
 *     function, fused                                                             -> reaxmoe_router_topk
 *   - the decision forward's element-wise steps around the MoE block (Gemma4DecoderLayer.forward, gemma4.py:696-771:
 *     RMSNorm + bf16 adds, q/k/v norms + RoPE, GELU-tanh * up)  -> reaxmoe_rmsnorm, reaxmoe_qkv_norm_rope,
 *                                                                    reaxmoe_gelu_tanh_mul
 *   - get_cutlass_moe_mm_data / blink _fplan (champions/uid240/opt/blink/blink_moe.py:271-299)
 *                                                                                 -> reaxmoe_plan
 *   - scaled_fp4_experts_quant of the m rows + _tscatter (blink_moe.py:301-323, :402-421)
 *                                                                                 -> reaxmoe_permute_quant
 *   - w13 grouped GEMM + gelu_tanh/silu * up + NVFP4 quant (blink_moegemm.cu:472-934 MODE 1,
 *     engine/fp4_triton.py:54-65, :161-167)                                       -> reaxmoe_gemm_w13
 *   - w2 grouped GEMM (blink_moegemm.cu:1173-1197, bmoe69.cu:1186-1189)           -> reaxmoe_gemm_w2
 *   - combine / unpermute _tail (blink_moe.py:168-198, :423-428)                  -> reaxmoe_combine
 *   - engine/fp4.py::quantize_nvfp4 (values, e4m3 block scales, 128x4 atoms, engine/fp4.py:16-52) and
 *     engine/fp4_triton.py::nvfp4_quant_static (:129-135)                         -> reaxmoe_quantize
 *   - int nv4_gemm(...) / size_t nv4_ws(...) C-ABI convention
 *     (champions/uid240/opt/reax/engine/nv4_dispatch.cu:11-26)                    -> status codes, workspace query
 *
 * Data formats (engine/fp4.py layout):
 *   NVFP4 matrix [R, K]: packed e2m1 bytes [R, K/2] (low nibble = even column) + e4m3 block scales (one per
 *   16 elements) in 128x4 atoms: byte (r, kb) lives at ((r/128)*(K/64) + kb/4)*512 + (r%32)*16 + ((r%128)/32)*4
 *   + kb%4. Weights are stacked per expert: w_fp4 [E, N, K/2], w_sf [E][N/128][K/64][512].
 *   Global scales: a*_gscale are QUANT-side (1 / dequant scale, vLLM convention); w*_alphas[e] = weight
 *   dequant scale x input dequant scale.
 *   Routed rows (vLLM layout): slot s of expert e is row expert_offsets[e] + i; its scale row is
 *   blockscale_offsets[e] + i (each expert's scale rows start on a 128-row atom).
 *   Slot order inside an expert is canonical: by (token, k-index) ascending.
 */
#ifndef REAXMOE_H
#define REAXMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  REAXMOE_OK = 0,
  REAXMOE_ERR_BAD_SHAPE = 1,       /* a size breaks a precondition (see reaxmoe_problem) */
  REAXMOE_ERR_MISALIGNED = 2,      /* a pointer is not 16-byte aligned */
  REAXMOE_ERR_TOO_MANY_EXPERTS = 3,/* experts > 256 or topk > 16 or topk > experts */
  REAXMOE_ERR_DEVICE_TIMEOUT = 4,  /* a bounded device wait expired (read back by reaxmoe_read_status) */
  REAXMOE_ERR_WORKSPACE = 5,       /* workspace NULL or smaller than reaxmoe_workspace_size() */
  REAXMOE_ERR_CUDA = 6,            /* a CUDA runtime / driver call failed */
  REAXMOE_ERR_NULL = 7,            /* a required pointer is NULL */
  REAXMOE_ERR_BAD_EXPERT_ID = 8,   /* a routed expert id >= experts (device-detected; negative ids mark unused slots) */
  REAXMOE_ERR_UNSUPPORTED = 9      /* e.g. no sm_100 device */
};

enum { REAXMOE_ACT_SILU = 0, REAXMOE_ACT_GELU_TANH = 1 };

/* Layer shape. vLLM names in brackets. Preconditions: hidden [k] % 128 == 0 in [256, 3072]; inter [n] % 64 == 0
 * in [256, 3072] (a GEMM m-tile's activation scales stay resident in tensor memory); 1 <= experts [e] <= 256;
 * 1 <= topk <= min(16, experts); tokens [m] >= 0. */
typedef struct reaxmoe_problem {
  int32_t tokens;
  int32_t hidden;
  int32_t inter;
  int32_t experts;
  int32_t topk;
  int32_t activation; /* REAXMOE_ACT_* */
} reaxmoe_problem;

typedef struct reaxmoe_forward_args {
  reaxmoe_problem p;
  const void* a;              /* [tokens, hidden] bf16 */
  const float* a1_gscale;     /* [experts] quant-side input scale of w13 */
  const void* w1_fp4;         /* [experts, 2*inter, hidden/2] u8, gate/up INTERLEAVED (reaxmoe_prepack_w13) */
  const void* w1_sf;          /* scale atoms of the interleaved w1_fp4, as reaxmoe_prepack_w13 writes them */
  const float* w1_alphas;     /* [experts] */
  const float* a2_gscale;     /* [experts] quant-side scale of the intermediate */
  const void* w2_fp4;         /* [experts, hidden, inter/2] u8 */
  const void* w2_sf;          /* scale atoms of w2_fp4 as engine/fp4.py lays them out: [experts][hidden/128][inter/64][512] */
  const float* w2_alphas;     /* [experts] */
  const float* topk_weights;  /* [tokens, topk] fp32 */
  const int32_t* topk_ids;    /* [tokens, topk] int32; a negative id marks an unused slot (contributes nothing) */
  void* output;               /* [tokens, hidden] bf16, written (not accumulated) */
} reaxmoe_forward_args;

/* Bytes of workspace reaxmoe_forward needs for this problem (0 on a bad shape). */
size_t reaxmoe_workspace_size(const reaxmoe_problem* p);

/* The whole layer: plan -> permute_quant -> gemm_w13 -> gemm_w2 -> combine
 * (run_cutlass_moe_fp4, cutlass_moe.py:481-664; blink_moe.py:434-567). When every expert has the same input scale
 * (a1_gscale), each token row is quantised once and w13 reads its A rows through the slot -> token map (the
 * gather layout of reaxmoe_permute_quant with rep_fp4 == NULL); otherwise the rows are replicated per slot. */
int reaxmoe_forward(const reaxmoe_forward_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* The same layer on token rows quantised upstream (reaxmoe_rmsnorm_nvfp4; the quant-once path of
 * blink_moe.py:353-363 with the norm fused, engine/fp4_triton.py:68-90): args->a points to packed e2m1 rows
 * [tokens, hidden / 2], a_scales to their linear e4m3 block scales [tokens, hidden / 16], made with the quant-side
 * scale a_gscale. Every expert must quantise with that scale (a1_gscale[e] == a_gscale; a routed expert that differs
 * sets REAXMOE_ERR_UNSUPPORTED in the device status word). hidden a multiple of 256, <= 4096. Same output as
 * reaxmoe_forward on the bf16 rows those bytes were made from. */
int reaxmoe_forward_prequant(const reaxmoe_forward_args* args, const void* a_scales, float a_gscale,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Gemma-4 routing: ids = top-k of logits (descending, ties to the lower expert id), weights = softmax over all
 * experts renormalised over the top-k, times per_expert_scale[id] (NULL = 1). logits [tokens, experts] fp32;
 * ids [tokens, topk] int32; weights [tokens, topk] fp32. (gemma4.py:183-203) */
int reaxmoe_route(const float* logits, const float* per_expert_scale, int32_t tokens, int32_t experts,
                  int32_t topk, int32_t* topk_ids, float* topk_weights, void* stream);

/* Caps the grid of this library's persistent kernels (grouped GEMMs, router, combine) at `sms` CTAs, leaving the
 * other SMs free for kernels that run beside them -- e.g. the NCCL all-to-alls of an overlapped expert-parallel
 * exchange. 0 (the default) = every SM of the device. Process-wide; set it between calls, not during one. */
void reaxmoe_set_sm_budget(int32_t sms);

/* Gemma-4 router fused with its routing (Gemma4Router.forward, vllm/model_executor/models/gemma4.py:251-298, as the
 * champion's router GEMM champions/uid240/opt/blink/blink_rgemm.cu:44-56 runs it, followed by gemma4.py:183-203):
 * u = bf16(bf16(bf16(rmsnorm(x)) * bf16(hidden^-1/2)) * router_scale) with rmsnorm = x * rsqrt(mean(x^2) + eps) in
 * fp32 (no weight; vllm/ir/ops/layernorm.py:10-21), logits = u . router_weight^T (bf16 products, fp32 accumulation
 * on the tensor cores), then top-k and weights exactly as reaxmoe_route from those logits. The logits stay on chip;
 * pass a [tokens, experts] fp32 buffer as `logits` to also store them (NULL: not stored). hidden_states [tokens,
 * hidden] bf16; router_scale [hidden] bf16; router_weight [experts, hidden] bf16; experts 32, 64 or 128; hidden % 128
 * == 0, <= 3072. `status` (NULL-able) receives REAXMOE_ERR_DEVICE_TIMEOUT if a bounded device wait expires. */
int reaxmoe_router_topk(const void* hidden_states, const void* router_scale, const void* router_weight,
                        const float* per_expert_scale, float eps, int32_t tokens, int32_t hidden, int32_t experts,
                        int32_t topk, int32_t* topk_ids, float* topk_weights, float* logits, int32_t* status,
                        void* stream);

/* ---- The decision forward's fused element-wise steps (the Gemma-4 layer around the MoE block,
 * vllm/model_executor/models/gemma4.py:696-771), each at vLLM's bf16 rounding points. All tensors bf16, contiguous,
 * 16-byte aligned; stream-ordered.
 *
 * out = bf16(bf16(s * rsqrt(mean(s^2) + eps)) * weight) [+ residual] with s = bf16(a [+ b]) (vLLM rms_norm,
 * vllm/ir/ops/layernorm.py:10-21, plus the bf16 adds around it). b, weight, residual may be NULL (weight NULL: no
 * scale). rows x cols, cols a multiple of 256 and <= 4096. */
int reaxmoe_rmsnorm(const void* a, const void* b, const void* weight, const void* residual, float eps, int64_t rows,
                    int32_t cols, void* out, void* stream);
/* reaxmoe_rmsnorm followed by the static NVFP4 quantisation of its bf16 output with the quant-side global scale
 * `gscale` (1 / g): packed [rows, cols / 2] e2m1 (low nibble = even column) and linear e4m3 block scales
 * [rows, cols / 16], the bytes permute_quant would make from the bf16 output (the add + RMSNorm + quant fusion of
 * engine/fp4_triton.py:68-90, with vLLM's norm arithmetic). `out` (bf16, NULL-able) receives the bf16 output too.
 * Feeds reaxmoe_forward_prequant. */
int reaxmoe_rmsnorm_nvfp4(const void* a, const void* b, const void* weight, const void* residual, float eps,
                          int64_t rows, int32_t cols, float gscale, void* out, void* packed, void* scales,
                          void* stream);
/* qkv [tokens, (q_heads + 2 kv_heads) * head_dim] -> q [tokens, q_heads, head_dim], k, v [tokens, kv_heads,
 * head_dim]: per-head RMSNorm of q and k with their weights [head_dim], of v without (Gemma4Attention.forward,
 * gemma4.py:512-535), then NeoX rotate-half of q and k with bf16 tables cos / sin [max_position, head_dim / 2]
 * indexed by positions [tokens] (int64), one bf16 rounding per operation (rotary_embedding/base.py). head_dim 64,
 * 128 or 256. */
int reaxmoe_qkv_norm_rope(const void* qkv, const void* q_weight, const void* k_weight, const void* cos_table,
                          const void* sin_table, const int64_t* positions, float eps, int64_t tokens, int32_t q_heads,
                          int32_t kv_heads, int32_t head_dim, void* q, void* k, void* v, void* stream);
/* gate_up [rows, 2 inter] -> out [rows, inter] = bf16(bf16(gelu_tanh(gate)) * up) (GeluAndMul native form). */
int reaxmoe_gelu_tanh_mul(const void* gate_up, int64_t rows, int32_t inter, void* out, void* stream);

/* Routing data (get_cutlass_moe_mm_data; blink_moe.py:271-299). Writes, inside the workspace, the per-expert
 * counts, expert_offsets[E+1], blockscale_offsets[E+1] and GEMM tile tables, and copies them out to the
 * optional (NULL-able) host-visible-or-device arrays given. */
int reaxmoe_plan(const reaxmoe_problem* p, const int32_t* topk_ids, void* workspace, size_t workspace_bytes,
                 int32_t* expert_offsets, int32_t* blockscale_offsets, int32_t* problem_sizes1,
                 int32_t* problem_sizes2, void* stream);

/* Quantise every token row once per distinct expert scale and scatter it to its top-k slots (FP4 rows +
 * swizzled scales) in the canonical order; writes c_map[t*topk + j] = slot (blink_moe.py:301-323). Needs the
 * plan of the same workspace. rep_fp4 [tokens*topk, hidden/2]; rep_sf scale atoms over blockscale_offsets.
 * rep_fp4 == NULL selects the gather layout (the reference's gather-A path, blink_moegemm.cu:532-647): when every
 * expert has the same a1_gscale, each token row is quantised once into the workspace, token-major, with a
 * slot -> token map beside it; when the scales differ, the per-slot rows go to the workspace instead. rep_sf and
 * c_map are written either way. reaxmoe_gemm_w13 with rep_fp4 == NULL then reads the layout this call chose. */
int reaxmoe_permute_quant(const reaxmoe_problem* p, const void* a, const float* a1_gscale, const int32_t* topk_ids,
                          void* workspace, size_t workspace_bytes, void* rep_fp4, void* rep_sf, int32_t* c_map,
                          void* stream);

/* Grouped NVFP4 GEMM w13 with the fused activation(gate) * up and NVFP4 re-quantisation epilogue
 * (blink_moegemm.cu:472-934 MODE 1). Needs the plan of the same workspace. w1_fp4 is interleaved
 * (reaxmoe_prepack_w13) with its scale atoms. hidden <= 3072. rep_fp4 == NULL: A rows from the gather layout that
 * reaxmoe_permute_quant (rep_fp4 == NULL) left in the same workspace. */
int reaxmoe_gemm_w13(const reaxmoe_problem* p, const void* rep_fp4, const void* rep_sf, const void* w1_fp4,
                     const void* w1_sf, const float* w1_alphas, const float* a2_gscale, void* workspace,
                     size_t workspace_bytes, void* int_fp4, void* int_sf, void* stream);

/* Grouped NVFP4 GEMM w2: c3[slot] = bf16(alpha_e * int[slot] . w2_e^T) (blink_moegemm.cu:1173-1197). w2_sf: the
 * engine/fp4.py scale atoms of w2_fp4 as they are. inter <= 3072. */
int reaxmoe_gemm_w2(const reaxmoe_problem* p, const void* int_fp4, const void* int_sf, const void* w2_fp4,
                    const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes, void* c3,
                    void* stream);

/* out[t] = bf16( sum_j bf16(c3[c_map[t*topk+j]] * bf16(w[t, j])) ), fp32 sums in the canonical order
 * ((s0 + s1) + s2) + s3 of 4 strided partial sums (blink_moe.py:168-198, ORDER 1 for top-8). A pair with
 * c_map -1 (no slot) adds exactly +0, whatever its weight. */
int reaxmoe_combine(const reaxmoe_problem* p, const void* c3, const int32_t* c_map, const float* topk_weights,
                    void* output, void* stream);

/* NVFP4 quantisation of rows (engine/fp4.py::quantize_nvfp4 numerics with a given scale; fp4_triton.py
 * nvfp4_quant_static). x [rows, cols] bf16 (x_is_fp32 = 0) or fp32 (1); rows are grouped by group_rows
 * (e.g. one expert's N rows), group g quantised with dequant scale 1 / gscale[g]; packed [rows, cols/2];
 * scales in 128x4 atoms, each group starting on its own atom row: scale row = (r / group_rows) *
 * ceil128(group_rows) + r % group_rows. cols % 64 == 0. */
int reaxmoe_quantize(const void* x, int32_t x_is_fp32, int64_t rows, int32_t cols, int32_t group_rows,
                     const float* gscale, void* packed, void* scales, void* stream);

/* One-time re-layout of w13 for the fused gate/up epilogue: output row block b (256 rows) = gate rows
 * [128b, 128b+h) then up rows inter + [128b, 128b+h), h = min(128, inter - 128b) (the last block is narrower when
 * inter % 128 != 0); scales move with their rows. In-place is NOT allowed. */
int reaxmoe_prepack_w13(const void* w1_fp4, const void* w1_sf, int32_t experts, int32_t inter, int32_t hidden,
                        void* w1p_fp4, void* w1p_sf, void* stream);

/* The routing-data plan of reaxmoe_plan for callers that cannot allocate device memory (no counterpart in the
 * reference). Same outputs as reaxmoe_plan (expert_offsets, blockscale_offsets and the optional problem sizes),
 * but no caller workspace: its scratch is a file-scope static device array of about 1 MiB that every GPU loading
 * this library holds until exit. Limit: tokens <= 65536 (REAXMOE_ERR_BAD_SHAPE beyond). The first call on a device
 * looks up the array's device address (cudaGetSymbolAddress) and should come before any stream capture. All calls
 * share the array, so calls that overlap on the GPU (e.g. on two streams) race. Routed ids outside [0, experts) are
 * skipped as in reaxmoe_plan, but this entry point reports no device status for them (there is no workspace to
 * hold the status word reaxmoe_read_status reads). Shapes are checked as in reaxmoe_plan. Allocates nothing (no
 * cudaMalloc / cudaFree). */
int reaxmoe_plan_static(const reaxmoe_problem* p, const int32_t* topk_ids, int32_t* expert_offsets,
                        int32_t* blockscale_offsets, int32_t* problem_sizes1, int32_t* problem_sizes2, void* stream);

/* ---- Expert parallelism (no counterpart in the reference, which requires ep_size == 1 at
 * champions/uid240/opt/blink/blink_par.py:99). The three calls below are the device halves of vLLM's
 * FusedMoEPrepareAndFinalize.prepare / finalize (vllm/model_executor/layers/fused_moe/modular_kernel.py:263-378;
 * naive form prepare_finalize/naive_dp_ep.py:112-209) around the grouped GEMMs; the caller moves the records with
 * two all-to-alls (NCCL). Rank r of `ranks` owns experts [r * El, (r + 1) * El), El = experts / ranks.
 *
 * Record (reaxmoe_ep_record_bytes(hidden, topk) bytes, a multiple of 16), one per (token, rank owning >= 1 of its
 * experts): [0, H/2) NVFP4 codes; [H/2, H/2 + H/16) e4m3 block scales, linear; then int32 local expert ids [topk]
 * (-1 for experts on other ranks) and fp32 router weights [topk]; zero or more padding bytes. */
size_t reaxmoe_ep_record_bytes(int32_t hidden, int32_t topk);

/* Dispatch: p describes this rank's tokens with the GLOBAL expert count. Writes send_counts [ranks] (records per
 * destination rank), the records grouped by destination rank in rank order and token order inside a rank
 * (send_records: capacity tokens * min(ranks, topk) records), and send_map [tokens, topk]: the record index of the
 * first pair j of a token on each destination rank, -1 elsewhere. The row is quantised with the destination's input
 * scale; a1_gscale [experts] must be constant over each rank's experts (device status REAXMOE_ERR_UNSUPPORTED
 * otherwise). 1 <= ranks <= 64, experts % ranks == 0. */
size_t reaxmoe_ep_dispatch_workspace_size(const reaxmoe_problem* p, int32_t ranks);
int reaxmoe_ep_dispatch(const reaxmoe_problem* p, int32_t ranks, const void* a, const float* a1_gscale,
                        const int32_t* topk_ids, const float* topk_weights, void* workspace, size_t workspace_bytes,
                        int32_t* send_counts, int32_t* send_map, void* send_records, void* stream);

/* Receiver: `local` has tokens = received records, experts = El (topk may exceed El). Runs plan, permute, the two
 * grouped GEMMs on this rank's expert weights (the same formats as reaxmoe_forward_args; alphas and a2_gscale are
 * the local [El] slices) and writes partial [tokens, hidden] bf16: per record, the combine of its local pairs
 * (the single-GPU combine order with the other ranks' pairs left out). */
size_t reaxmoe_ep_expert_workspace_size(const reaxmoe_problem* local);
int reaxmoe_ep_expert_forward(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                              const void* w1_sf, const float* w1_alphas, const float* a2_gscale, const void* w2_fp4,
                              const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes,
                              void* partial, void* stream);

/* Source-side combine: output[t] = bf16( sum over j = 0..topk-1 with send_map[t, j] >= 0 of
 * float(returned[send_map[t, j]]) ), summed in fp32 from +0 in increasing j. returned [sum(send_counts), hidden]
 * bf16 holds the partial rows in send-record order (the reverse all-to-all of reaxmoe_ep_expert_forward's output). */
int reaxmoe_ep_combine(int32_t tokens, int32_t hidden, int32_t topk, const int32_t* send_map, const void* returned,
                       void* output, void* stream);

/* ---- NVLink peer-memory transport of the expert-parallel layer: the same records and rows as above, but the
 * pack kernel and the receiver's pre-sum kernel store them straight into the destination rank's buffers (CUDA IPC
 * mappings of the peers' memory over NVLink; no NCCL on the data path, no multicast). It replaces the two
 * all-to-alls of vLLM's naive EP prepare / finalize (prepare_finalize/naive_dp_ep.py:112-209). One forward on rank r:
 *   reaxmoe_ep_dispatch_plan -> send_counts; reaxmoe_ep_signal(epoch e, send_counts) -> every rank's count matrix;
 *   read it on the host; reaxmoe_ep_dispatch_pack (records into the peers); reaxmoe_ep_signal(e + 1);
 *   reaxmoe_ep_expert_forward_to (rows into the sources); reaxmoe_ep_signal(e + 2); reaxmoe_ep_combine. */

/* Device memory that peers can map: cudaMalloc'd, zeroed, with its 64-byte CUDA IPC handle in `handle`. */
int reaxmoe_ipc_alloc(size_t bytes, void** ptr, void* handle);
/* Maps a peer's reaxmoe_ipc_alloc memory (its handle) into this process; unmap with reaxmoe_ipc_close. */
int reaxmoe_ipc_open(const void* handle, void** ptr);
int reaxmoe_ipc_close(void* ptr);
int reaxmoe_ipc_free(void* ptr);

/* Signal block: bytes of each rank's block (from reaxmoe_ipc_alloc). Layout: int32 status at 0 (read it with
 * reaxmoe_read_status), uint32 flags [64] at 256 (flag s written by rank s), int32 send-count matrix [64][64] at 512
 * (row s = rank s's send_counts). */
size_t reaxmoe_ep_signal_bytes(void);
/* Cross-rank signal on `stream`: blocks [ranks] = every rank's signal block as mapped in this process (this rank's
 * own at index rank). With send_counts (device [ranks]) it first writes them into row `rank` of every rank's count
 * matrix. Then it sets flag `rank` of every block to `epoch` (after a system-scope fence that covers the earlier
 * kernels of the stream) and waits until all of this rank's flags reach `epoch`, at most timeout_ns; a wait that
 * runs out sets the block's status to REAXMOE_ERR_DEVICE_TIMEOUT. All ranks call it in the same order with the same
 * epochs (start at 1, one more per call). */
int reaxmoe_ep_signal(int32_t ranks, int32_t rank, const uint64_t* blocks, uint32_t epoch,
                      const int32_t* send_counts, uint64_t timeout_ns, void* stream);

/* reaxmoe_ep_dispatch's routing steps alone: send_counts [ranks] and the plan in `workspace`
 * (reaxmoe_ep_dispatch_workspace_size bytes). */
int reaxmoe_ep_dispatch_plan(const reaxmoe_problem* p, int32_t ranks, const float* a1_gscale,
                             const int32_t* topk_ids, void* workspace, size_t workspace_bytes, int32_t* send_counts,
                             void* stream);
/* The pack after reaxmoe_ep_dispatch_plan on the same workspace: writes send_map as reaxmoe_ep_dispatch does and
 * the records for rank d at records[d] (host array [ranks] of device addresses, 16-byte aligned: this rank's first
 * record in rank d's receive buffer, i.e. base_d + rec_bytes * sum_{s < r} counts[s][d]). */
int reaxmoe_ep_dispatch_pack(const reaxmoe_problem* p, int32_t ranks, const void* a, const float* a1_gscale,
                             const int32_t* topk_ids, const float* topk_weights, const void* workspace,
                             size_t workspace_bytes, int32_t* send_map, const uint64_t* records, void* stream);
/* reaxmoe_ep_expert_forward with the pre-summed row of received record i stored at
 * rows[s] + (i - bounds[s]) * hidden * 2 for the source s with bounds[s] <= i < bounds[s + 1] (host arrays:
 * bounds [ranks + 1] from 0 to local->tokens, non-decreasing; rows [ranks] device addresses, 32-byte aligned:
 * the row in rank s's return buffer of the first record s sent here). Every record's row is stored by the pre-sum
 * kernel. With environment REAXMOE_EP_DIRECT_ROWS=1 (read once per process) a record with
 * exactly one local pair gets its row from the w2 GEMM's epilogue instead; the rows are bit-identical either way,
 * signed zeros included, for router weights of any sign. */
int reaxmoe_ep_expert_forward_to(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                                 const void* w1_sf, const float* w1_alphas, const float* a2_gscale,
                                 const void* w2_fp4, const void* w2_sf, const float* w2_alphas, void* workspace,
                                 size_t workspace_bytes, int32_t ranks, const int64_t* bounds, const uint64_t* rows,
                                 void* stream);

/* reaxmoe_ep_expert_forward_to in two calls, so that the row stores of one part of the received records can run
 * beside the GEMMs of the next part (no counterpart in the reference). ep_expert_gemms: unpack, plan, permute and
 * the two grouped GEMMs of `local` (the part's records), with c3 left in `workspace`
 * (reaxmoe_ep_expert_workspace_size(local) bytes, one workspace per part in flight); its persistent GEMMs use at
 * most sm_limit SMs (0 = all). ep_presum_to: then, on any stream ordered after it, the pre-summed row of each of the
 * part's records stored as reaxmoe_ep_expert_forward_to stores it (bounds / rows relative to the part), by one
 * 1024-thread block per SM on `sms` SMs (0 = the plain launch on every SM). */
int reaxmoe_ep_expert_gemms(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                            const void* w1_sf, const float* w1_alphas, const float* a2_gscale, const void* w2_fp4,
                            const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes,
                            int32_t sm_limit, void* stream);
int reaxmoe_ep_presum_to(const reaxmoe_problem* local, const void* workspace, size_t workspace_bytes, int32_t ranks,
                         const int64_t* bounds, const uint64_t* rows, int32_t sms, void* stream);

/* n device-to-device copies on `stream`, dst[i] <- src[i] (bytes[i] each; host arrays of device addresses), one
 * cudaMemcpyAsync each: the copy engines move them, over NVLink when a destination is a peer's CUDA-IPC-mapped
 * buffer, without taking SMs from the kernels running beside them. Used to return one part's pre-summed rows from a
 * local staging buffer to their source ranks while the next part's GEMMs run (no counterpart in the reference). */
int reaxmoe_ep_copy_rows(int32_t n, const uint64_t* dst, const uint64_t* src, const uint64_t* bytes, void* stream);

/* Synchronises `stream`, returns the device status word of the workspace (0 = ok, else REAXMOE_ERR_*) and
 * clears it when `clear` != 0. Not for the hot path. */
int reaxmoe_read_status(void* workspace, size_t workspace_bytes, int32_t clear, void* stream);

/* Copies the last error text of the calling thread into buf (NUL-terminated); returns its full length. */
size_t reaxmoe_last_error(char* buf, size_t len);

/* Library version (major * 10000 + minor * 100 + patch). */
int32_t reaxmoe_version(void);

#ifdef __cplusplus
}
#endif

#endif /* REAXMOE_H */
