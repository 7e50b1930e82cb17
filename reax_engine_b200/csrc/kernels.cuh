// kernels.cuh -- host launchers of the routing / permute / combine / quantise / prepack kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace reaxmoe {

int launch_route(const float* logits, const float* scale, int T, int E, int K, int* ids, float* w, cudaStream_t s);
int launch_count(const int* ids, int m, int k, int E, int* seg_counts, int* status, cudaStream_t s);
int launch_plan(const int* seg_counts, int nseg, int E, int* seg_base, int* counts, int* eoff, int* boff,
                int* tile_prefix, int* ps1, int* ps2, int n1, int k1, int n2, int k2, cudaStream_t s);
// The permute kernels write scale bytes to a linear buffer lin_sf [slots, H/16]; launch_swizzle_scales then writes
// the 128x4 atoms of every m-tile (needs the plan's tile_prefix / counts / expert_offsets).
// The gather layout of the w13 A operand: token-major FP4 rows and scale rows, quantised once per token, and the
// slot -> token map through which the GEMM and the scale swizzle read them. flag (one int, written by the permute
// stage) says whether the token-major layout was written (1) or, because the experts' input scales differ, the
// per-slot rows (0).
struct GatherRows {
  uint8_t* tok_fp4;   // [tokens, H/2]
  uint8_t* tok_sf;    // [tokens, H/16]
  int* row_token;     // [slots]
  int* flag;
};
int launch_permute_quant(const __nv_bfloat16* a, const float* a1_gscale, const int* ids, const int* seg_base,
                         const int* eoff, const int* boff, int m, int H, int E, int k, uint8_t* rep_fp4,
                         uint8_t* lin_sf, int* c_map, cudaStream_t s, const GatherRows* ga = nullptr);
int launch_swizzle_scales(const uint8_t* lin, const int* tile_prefix, const int* counts, const int* eoff, int E, int H,
                          int64_t slots, uint8_t* sf, cudaStream_t s, const int* row_map = nullptr,
                          const int* ga_flag = nullptr, const uint8_t* tok_sf = nullptr, int tok_rows = 0,
                          int64_t tok_stride = 0);
int launch_combine(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                   __nv_bfloat16* out, int num_sms, cudaStream_t s);
int launch_quantize(const void* x, bool f32, int64_t rows, int cols, int group_rows, const float* gscale,
                    uint8_t* packed, uint8_t* scales, cudaStream_t s);
int launch_prepack_w13(const uint8_t* w, const uint8_t* sf, int E, int inter, int H, uint8_t* wp, uint8_t* sfp,
                       cudaStream_t s);

// Expert-parallel dispatch / receive / combine (ep.cu).
int launch_ep_rank_ids(const int* ids, int m, int k, int E, int El, const float* a1_gscale, int* rid, int* status,
                       cudaStream_t s);
int launch_ep_pack(const __nv_bfloat16* a, const float* a1_gscale, const int* ids, const float* w, const int* rid,
                   const int* seg_base, const int* roff, int m, int H, int E, int El, int k, int rec_bytes,
                   uint8_t* records, int* send_map, cudaStream_t s);
int launch_ep_unpack_meta(const uint8_t* records, int n, int k, int H, int rec_bytes, int* lid, float* lw,
                          cudaStream_t s);
int launch_ep_permute(const uint8_t* records, const int* lid, const int* seg_base, const int* eoff, int n, int H,
                      int El, int k, int rec_bytes, uint8_t* rep_fp4, uint8_t* lin_sf, int* c_map, cudaStream_t s,
                      const GatherRows* ga = nullptr);
int launch_ep_combine(const __nv_bfloat16* ret, const int* map, int m, int H, int k, __nv_bfloat16* out, int num_sms,
                      cudaStream_t s);

// Peer-memory (NVLink) transport of the expert-parallel layer. Addresses are device virtual addresses valid in this
// process: this GPU's own buffers or peers' buffers mapped through CUDA IPC.
struct PeerPtrs {
  uint64_t p[kMaxRanks];
};
// Destination of the pre-summed row of received record i: rows.p[s] + (i - bound[s]) * row_bytes for the source s
// with bound[s] <= i < bound[s + 1].
struct RowRoute {
  uint64_t p[kMaxRanks];
  int64_t bound[kMaxRanks + 1];
  int ranks;
  int skip_single;  // the combine leaves out records with exactly one local pair (the w2 epilogue sent those)
#ifdef __CUDACC__
  __device__ __forceinline__ uint64_t row_addr(int64_t t, int H) const {
    int src = 0;
    for (int q = 1; q < ranks; ++q) src += (t >= bound[q]) ? 1 : 0;
    return p[src] + (uint64_t)(t - bound[src]) * (uint64_t)H * 2u;
  }
#endif
};
// Signal block (one per rank, peer-mapped): status word, one flag per source rank, the [ranks, ranks] send-count
// matrix (row s written by rank s).
constexpr int kSigStatus = 0;
constexpr int kSigFlags = 256;
constexpr int kSigCounts = 512;
constexpr size_t kSigBytes = 512 + 4 * kMaxRanks * kMaxRanks;
// pack with records[d] = address of this rank's first record in rank d's receive buffer
int launch_ep_pack_peer(const __nv_bfloat16* a, const float* a1_gscale, const int* ids, const float* w, const int* rid,
                        const int* seg_base, const int* roff, int m, int H, int E, int El, int k, int rec_bytes,
                        const PeerPtrs& records, int* send_map, cudaStream_t s);
int launch_combine_routed(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                          const RowRoute& route, int num_sms, cudaStream_t s);
int launch_combine_routed_pinned(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                                 const RowRoute& route, int sms, cudaStream_t s);
int launch_ep_signal(const PeerPtrs& blocks, int rank, int ranks, uint32_t epoch, const int* counts,
                     unsigned long long timeout_ns, cudaStream_t s);
// Direct rows: for every received record with exactly one local pair, its slot's entry gets the record's return
// address (route) and router weight; the other local pairs' slots get 0 (summed by the routed combine).
int launch_ep_direct(const int* c_map, const float* lw, int n, int k, int H, const RowRoute& route,
                     uint64_t* direct_dst, float* direct_w, cudaStream_t s);

// Grouped NVFP4 GEMM (gemm_sm100.cu). mode 0: out bf16 [slots, N]; mode 1: fused act(gate)*up + NVFP4 quant
// into q_out [slots, N/4] (N = 2*inter interleaved) and q_sf atoms.
struct GemmLaunch {
  int mode;          // 0 = plain (w2), 1 = w13 fused
  int act;           // REAXMOE_ACT_*
  const void* a;     // [slots, K/2]
  int64_t slots;
  const void* a_sf;  // atoms over blockscale rows
  const void* b;     // [E, N, K/2]
  const void* b_sf;  // weight scale atoms as engine/fp4.py lays them out: [E][N/128][K/64][512]
  const float* alphas;
  int E, N, K;
  const int* counts; const int* eoff; const int* boff; const int* tile_prefix;
  void* out;         // mode 0: bf16 [slots, N]
  void* q_out;       // mode 1: [slots, N/4]
  void* q_sf;        // mode 1: atoms over blockscale rows, K/64 = (N/2)/64 atom columns
  const float* q_gscale;
  int* status;
  unsigned long long timeout_ns;
  // mode 1, gather layout (row_token != nullptr): A rows are read through the slot -> token map from a_tok
  // [tokens, K/2] when *ga_flag is set, else from the per-slot rows at `a` (the permute stage decides)
  const void* a_tok;
  const int* row_token;
  const int* ga_flag;
  int64_t tokens;
  int64_t tok_stride;   // bytes between consecutive rows of a_tok (0: K/2, packed rows)
  // mode 0, expert-parallel receiver: slot rows whose direct_dst is non-zero are written as the record's finished
  // row, bf16(bf16(alpha * acc) * bf16(direct_w)) (+0 normalised when topk > 1, as the combine's sum does), at
  // direct_dst (a peer's return buffer over NVLink) instead of c3
  const uint64_t* direct_dst;
  const float* direct_w;
  int topk;
};
int launch_grouped_gemm(const GemmLaunch& g, int num_sms, cudaStream_t s);

// Fused Gemma-4 router + top-k (router_sm100.cu).
struct RouterLaunch {
  const void* x;       // [T, H] bf16
  const void* scale;   // [H] bf16 learned router input scale
  const void* w;       // [E, H] bf16 router weight
  const float* pes;    // [E] per-expert scale of the routing weights, or null
  float root;          // bf16(H^-1/2) as a float
  float eps;
  int T, H, E, K;
  int* ids;            // [T, K]
  float* wts;          // [T, K]
  float* logits;       // optional [T, E] fp32
  int* status;
  unsigned long long timeout_ns;
  int num_sms;         // the persistent grid's upper bound
};
int launch_router_topk(const RouterLaunch& r, cudaStream_t s);

// decision_ops.cu: the decision forward's fused element-wise steps
int launch_rmsnorm(const void* a, const void* b, const void* w, const void* res, float eps, int64_t rows, int cols,
                   void* out, cudaStream_t s);
int launch_qkv_norm_rope(const void* qkv, const void* qw, const void* kw, const void* cos_t, const void* sin_t,
                         const int64_t* pos, float eps, int64_t n, int hq, int hk, int d, void* q, void* k, void* v,
                         cudaStream_t s);
int launch_gelu_tanh_mul(const void* gu, int64_t rows, int inter, void* h, cudaStream_t s);
int launch_rmsnorm_nvfp4(const void* a, const void* b, const void* w, const void* res, float eps, int64_t rows,
                         int cols, float gscale, void* out, uint8_t* packed, uint8_t* scales, cudaStream_t s);
int launch_permute_fp4(const uint8_t* a_fp4, const uint8_t* a_sf, float in_gscale, const float* a1_gscale,
                       const int* ids, const int* seg_base, const int* eoff, int m, int H, int E, int k,
                       uint8_t* rep_fp4, uint8_t* lin_sf, int* c_map, int* status, cudaStream_t s,
                       const GatherRows* ga = nullptr);

}  // namespace reaxmoe
