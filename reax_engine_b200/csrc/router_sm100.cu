// router_sm100.cu -- the Gemma-4 router fused with its top-k routing: router logits are computed on the tensor
// cores (tcgen05, bf16 operands, fp32 accumulation in TMEM) and the top-k / renormalised weights are taken straight
// from TMEM, so the [tokens, experts] fp32 logits never reach HBM.
//
// Replaces the router projection of vLLM's Gemma4Router.forward (vllm/model_executor/models/gemma4.py:251-298) as
// run by the reference's champion router GEMM (champions/uid240/opt/blink/blink_rgemm.cu:44-56, blink_rtr.py:4-8),
// followed by the Gemma-4 routing function (gemma4.py:183-203). Same arithmetic per token:
//   r   = 1 / sqrt(mean_h(x_h^2) + eps)                     (fp32; vllm/ir/ops/layernorm.py:10-21, no weight)
//   u_h = bf16(bf16(bf16(x_h * r) * bf16(hidden^-1/2)) * bf16(scale_h))
//   logit_e = sum_h u_h * W[e, h]                           (bf16 x bf16 products, fp32 accumulation)
//   ids = top-k of the logits (larger first, ties to the lower expert id); weights = softmax over the top-k,
//   times per_expert_scale[id] -- exactly as reaxmoe_route computes them from the same logits.
//
// Design: a persistent kernel, one CTA per SM, each taking 128-token tiles in turn. A tile is read twice, through
// two rings of shared-memory slots fed by two TMA producers: ring 1 carries its x chunks [128 tokens x 64] for pass
// 1 (from HBM, evict_last), ring 2 the same x chunks again with the router weight chunks [E x 64] for pass 2 (from L2,
// evict_first). Pass 1 runs one tile ahead of pass 2, so HBM streams the next tile while the current one is being
// multiplied.
//   warp 0       ring-1 producer          warp 2   ring-2 producer (128-byte swizzle; rows past the last token are
//                                                  zero-filled by TMA)
//   warp 1       allocates E columns of TMEM; one thread issues tcgen05.mma.kind::f16 (M = 128, N = E, K = 16).
//   warps 4..7   pass 1: thread = row; the row's sum of squares in fp32, in ascending column order; then
//                r = rsqrt(mean + eps) into a double-buffered per-row array.
//   warps 8..15  pass 2: thread (row r = tid / 2, half h = tid % 2) rewrites its four 16-byte pieces of every chunk
//                in place as u -- the swizzle keeps a token's 64 elements inside its own 128-byte row, so the
//                element-wise transform leaves every piece where the MMA expects it.
//   warps 16..19 epilogue, one warp per TMEM lane quarter: each thread reads its token's E logits from TMEM 32
//                columns at a time into a running sorted top-k list, releases TMEM, and writes ids and weights.
// All waits are bounded (globaltimer); a timeout records REAXMOE_ERR_DEVICE_TIMEOUT and the CTA winds down.
#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace reaxmoe {
namespace router {

using namespace sm100;

constexpr int BM = 128;                        // tokens per tile (MMA M)
constexpr int KCH = 64;                        // bf16 elements per K chunk = one 128-byte swizzle row
constexpr int S1 = 3;                          // ring-1 slots (x tile, 16 KiB)
constexpr int S2 = 5;                          // ring-2 slots (x tile + weight tile, 32 KiB); pass 2 holds a
                                               // slot through TMA latency, transform and MMA: it gets the depth
constexpr int MAX_E = 128;
constexpr int A_BYTES = BM * KCH * 2;          // 16 KiB x tile
constexpr int B_BYTES = MAX_E * KCH * 2;       // 16 KiB weight tile
constexpr int R2_BYTES = A_BYTES + B_BYTES;
constexpr int P1W0 = 4, P1W = 4;               // pass-1 warps
constexpr int P2W0 = 8, P2W = 8;               // pass-2 warps
constexpr int EW0 = 16;                        // epilogue warps 16..19
constexpr int THREADS = (EW0 + 4) * 32;
constexpr int MAX_H = 3072;
constexpr int SMEM_BYTES = 1024 + S1 * A_BYTES + S2 * R2_BYTES + MAX_H * 2 + 2 * BM * 4 + 512;

// tcgen05.mma.kind::f16 instruction descriptor: fp32 accumulator (bit 4), A and B bf16 (bits 7, 10), both K-major,
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_bf16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// order-preserving map of a float to an unsigned key (-0.0 and +0.0 equal; 0 is below every key), and back
__device__ __forceinline__ uint32_t sort_key(float v) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Running top-KM list, sorted by key descending; a candidate enters strictly above every entry it beats, so among
// equal keys the one seen first (the lower expert id, candidates arrive in id order) stays ahead. Each entry moves
// down by at most one place per insertion, decided against the list before the insertion.
template <int KM>
__device__ __forceinline__ void topk_insert(uint32_t c, int ci, uint32_t (&lk)[KM], int (&li)[KM]) {
  bool g[KM];
#pragma unroll
  for (int j = 0; j < KM; ++j) g[j] = c > lk[j];
#pragma unroll
  for (int j = KM - 1; j > 0; --j) {
    lk[j] = g[j] ? (g[j - 1] ? lk[j - 1] : c) : lk[j];
    li[j] = g[j] ? (g[j - 1] ? li[j - 1] : ci) : li[j];
  }
  lk[0] = g[0] ? c : lk[0];
  li[0] = g[0] ? ci : li[0];
}

struct Params {
  CUtensorMap tmX;   // hidden states [T, H] bf16 as u8 [T, 2H], box 128 B x 128 rows, 128-byte swizzle
  CUtensorMap tmW;   // router weight [E, H] bf16 as u8 [E, 2H], box 128 B x E rows, 128-byte swizzle
  const __nv_bfloat16* scale;
  const float* pes;  // per-expert scale of the routing weights (nullable)
  float root;        // bf16(hidden^-1/2) as a float
  float eps;
  int T, H, E, K;
  int* ids;
  float* wts;
  float* logits;     // optional [T, E] fp32
  int* status;
  unsigned long long timeout_ns;
};

template <int E, int KM>
__global__ void __launch_bounds__(THREADS, 1) router_topk_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring1 = smem;                                  // S1 x tiles
  uint8_t* ring2 = smem + S1 * A_BYTES;                   // S2 (x tile, weight tile)
  __nv_bfloat16* sc_s = reinterpret_cast<__nv_bfloat16*>(ring2 + S2 * R2_BYTES);
  float* rsq_s = reinterpret_cast<float*>(sc_s + MAX_H);  // [2][BM]
  uint64_t* bars = reinterpret_cast<uint64_t*>(rsq_s + 2 * BM);
  uint64_t* full1 = bars;                // [S1] ring-1 tile landed (tx)
  uint64_t* empty1 = full1 + S1;         // [S1] pass 1 read the slot (one arrival per pass-1 warp)
  uint64_t* full2 = empty1 + S1;         // [S2] ring-2 tiles landed (tx)
  uint64_t* a_full = full2 + S2;         // [S2] the slot's x tile was rewritten as u (one arrival per pass-2 warp)
  uint64_t* empty2 = a_full + S2;        // [S2] the slot's MMAs completed (commit)
  uint64_t* rsq_full = empty2 + S2;      // [2] a tile's rsqrt values are in rsq_s[b] (one arrival per pass-1 warp)
  uint64_t* rsq_empty = rsq_full + 2;    // [2] pass 2 took its rsqrt values (one arrival per pass-2 warp)
  uint64_t* accf = rsq_empty + 2;        // a tile's MMAs completed: logits in TMEM (commit)
  uint64_t* tmem_free = accf + 1;        // the epilogue read the logits out of TMEM (one arrival per warp)
  uint64_t* drainb = tmem_free + 1;      // the MMA issuer's final commit
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drainb + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int H = p.H;
  const int n = H / KCH;                               // chunks per pass
  const int n_tiles = (p.T + BM - 1) / BM;
  constexpr int TMEM_COLS = E <= 32 ? 32 : (E <= 64 ? 64 : 128);

  for (int i = threadIdx.x; i < H; i += blockDim.x) sc_s[i] = p.scale[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < S1; ++s) {
      mbar_init(smem_u32(&full1[s]), 1);
      mbar_init(smem_u32(&empty1[s]), P1W);
    }
    for (int s = 0; s < S2; ++s) {
      mbar_init(smem_u32(&full2[s]), 1);
      mbar_init(smem_u32(&a_full[s]), P2W);
      mbar_init(smem_u32(&empty2[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&rsq_full[b]), P1W);
      mbar_init(smem_u32(&rsq_empty[b]), P2W);
    }
    mbar_init(smem_u32(accf), 1);
    mbar_init(smem_u32(tmem_free), 4);
    mbar_init(smem_u32(drainb), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmX)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmW)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ TMA producers (ring 1: warp 0, ring 2: warp 2)
    if (lane == 0) {
      const bool r1 = warp == 0;
      const int S = r1 ? S1 : S2;
      uint64_t* fullb = r1 ? full1 : full2;
      uint64_t* emptyb = r1 ? empty1 : empty2;
      const uint64_t keep = l2_evict_last(), drop = l2_evict_first();
      int g = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
        for (int kc = 0; kc < n; ++kc, ++g) {
          const int s = g % S;
          if (g >= S &&
              !wait_bounded(smem_u32(&emptyb[s]), (uint32_t)(g / S - 1) & 1u, abort_flag, p.status, p.timeout_ns)) {
            ok = false;
            break;
          }
          if (r1) {
            mbar_expect_tx(smem_u32(&full1[s]), (uint32_t)A_BYTES);
            tma_load_2d_hint(smem_u32(ring1 + s * A_BYTES), &p.tmX, smem_u32(&full1[s]), kc * KCH * 2, tile * BM,
                             keep);
          } else {
            uint8_t* slot = ring2 + s * R2_BYTES;
            mbar_expect_tx(smem_u32(&full2[s]), (uint32_t)(A_BYTES + E * KCH * 2));
            tma_load_2d_hint(smem_u32(slot), &p.tmX, smem_u32(&full2[s]), kc * KCH * 2, tile * BM, drop);
            tma_load_2d_hint(smem_u32(slot + A_BYTES), &p.tmW, smem_u32(&full2[s]), kc * KCH * 2, 0, keep);
          }
        }
      }
      // let the last loads land before the CTA may exit (only matters after an abort)
      for (int f = g - 1; f >= 0 && f >= g - S; --f)
        wait_drain(smem_u32(&fullb[f % S]), (uint32_t)(f / S) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(E);
      int g = 0;
      int lt = 0;                      // tiles done by this CTA
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++lt) {
        if (lt > 0 && !wait_bounded(smem_u32(tmem_free), (uint32_t)(lt - 1) & 1u, abort_flag, p.status,
                                    p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kc = 0; kc < n; ++kc, ++g) {
          const int s = g % S2;
          if (!wait_bounded(smem_u32(&a_full[s]), (uint32_t)(g / S2) & 1u, abort_flag, p.status, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_s = smem_u32(ring2 + s * R2_BYTES);
          const uint32_t b_s = a_s + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < KCH / 16; ++kk)
            tc_mma_bf16(tmem, desc_sw128(a_s + kk * 32), desc_sw128(b_s + kk * 32), idesc,
                        (kc | kk) != 0 ? 1u : 0u);
          tc_commit(smem_u32(&empty2[s]));
        }
        if (ok) tc_commit(smem_u32(accf));
      }
      // every issued MMA has completed before TMEM may be released (matters after an abort)
      tc_commit(smem_u32(drainb));
      wait_drain(smem_u32(drainb), 0);
    }
  } else if (warp >= P1W0 && warp < P1W0 + P1W) {
    // ------------------------------------------------------------------ pass 1: row sums of squares
    const int r = threadIdx.x - P1W0 * 32;       // 0..127
    const int sw = r & 7;
    int g = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++lt) {
      const int b = lt & 1;
      float ss = 0.0f;
      for (int kc = 0; kc < n; ++kc, ++g) {
        const int s = g % S1;
        if (!wait_bounded(smem_u32(&full1[s]), (uint32_t)(g / S1) & 1u, abort_flag, p.status, p.timeout_ns)) {
          ok = false;
          break;
        }
        const uint8_t* row = ring1 + s * A_BYTES + r * 128;
        uint4 v[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) v[c] = *reinterpret_cast<const uint4*>(row + ((c ^ sw) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&empty1[s]));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float f[8];
          bf16x8_to_f32(v[c], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss = __fmaf_rn(f[e], f[e], ss);   // f * f is exact: one rounding per step
        }
      }
      if (!ok) break;
      if (lt >= 2 && !wait_bounded(smem_u32(&rsq_empty[b]), (uint32_t)(lt / 2 - 1) & 1u, abort_flag, p.status,
                                   p.timeout_ns))
        break;
      rsq_s[b * BM + r] = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps));
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&rsq_full[b]));
    }
  } else if (warp >= P2W0 && warp < P2W0 + P2W) {
    // ------------------------------------------------------------------ pass 2: x tiles rewritten as u, in place
    const int tid = threadIdx.x - P2W0 * 32;     // 0..255
    const int r = tid >> 1, h = tid & 1;
    const int sw = r & 7;
    const __nv_bfloat162 root2 = __floats2bfloat162_rn(p.root, p.root);
    int g = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++lt) {
      const int b = lt & 1;
      if (!wait_bounded(smem_u32(&rsq_full[b]), (uint32_t)(lt / 2) & 1u, abort_flag, p.status, p.timeout_ns)) break;
      const float rs = rsq_s[b * BM + r];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&rsq_empty[b]));
      for (int kc = 0; kc < n; ++kc, ++g) {
        const int s = g % S2;
        if (!wait_bounded(smem_u32(&full2[s]), (uint32_t)(g / S2) & 1u, abort_flag, p.status, p.timeout_ns)) {
          ok = false;
          break;
        }
        uint8_t* row = ring2 + s * R2_BYTES + r * 128;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = h * 4 + j;                   // logical 16-byte chunk: columns kc * 64 + c * 8 .. + 7
          uint4* piece = reinterpret_cast<uint4*>(row + ((c ^ sw) << 4));
          const uint4 v = *piece;
          const uint4 scv = *reinterpret_cast<const uint4*>(sc_s + kc * KCH + c * 8);
          const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
          const uint32_t sw4[4] = {scv.x, scv.y, scv.z, scv.w};
          uint32_t o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // bf16(x * r) from the fp32 product; the two bf16 x bf16 products are exact before their one rounding
            const __nv_bfloat162 t1 = __floats2bfloat162_rn(__fmul_rn(__uint_as_float(xw[q] << 16), rs),
                                                            __fmul_rn(__uint_as_float(xw[q] & 0xFFFF0000u), rs));
            const __nv_bfloat162 t2 = __hmul2_rn(t1, root2);
            const __nv_bfloat162 u = __hmul2_rn(t2, *reinterpret_cast<const __nv_bfloat162*>(&sw4[q]));
            o[q] = *reinterpret_cast<const uint32_t*>(&u);
          }
          *piece = make_uint4(o[0], o[1], o[2], o[3]);
        }
        fence_async_smem();   // the generic-proxy stores above become visible to the tensor core's async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&a_full[s]));
      }
    }
  } else if (warp >= EW0) {
    // ------------------------------------------------------------------ epilogue: top-k from TMEM
    const int q = warp & 3;                      // TMEM lane quarter of this warp
    const int r = q * 32 + lane;
    int lt = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++lt) {
      if (!wait_bounded(smem_u32(accf), (uint32_t)lt & 1u, abort_flag, p.status, p.timeout_ns)) break;
      tc_fence_after();
      const int64_t t = (int64_t)tile * BM + r;
      const bool live = t < p.T;
      uint32_t lk[KM];
      int li[KM];
#pragma unroll
      for (int j = 0; j < KM; ++j) {
        lk[j] = 0u;
        li[j] = 0;
      }
#pragma unroll
      for (int c0 = 0; c0 < E; c0 += 32) {
        uint32_t v[32];
        tc_ld_32x32b_x32(tmem + ((uint32_t)(q * 32) << 16) + c0, v);
        tc_wait_ld();
        if (live && p.logits != nullptr) {
          float4* lrow = reinterpret_cast<float4*>(p.logits + t * E + c0);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            lrow[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                  __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t key = sort_key(__uint_as_float(v[i]));
          if (key > lk[KM - 1]) topk_insert<KM>(key, c0 + i, lk, li);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(tmem_free));
      if (live) {
        const float v0 = key_value(lk[0]);
        float ex[KM];
        float denom = 0.0f;
#pragma unroll
        for (int j = 0; j < KM; ++j) {
          ex[j] = expf(key_value(lk[j]) - v0);
          if (j < p.K) denom = __fadd_rn(denom, ex[j]);
        }
#pragma unroll
        for (int j = 0; j < KM; ++j) {
          if (j < p.K) {
            float w = __fdiv_rn(ex[j], denom);
            if (p.pes != nullptr) w = __fmul_rn(w, p.pes[li[j]]);
            p.ids[t * p.K + j] = li[j];
            p.wts[t * p.K + j] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

template <int E, int KM>
static int launch_e(const Params& prm, int grid, cudaStream_t s) {
  auto kfn = router_topk_kernel<E, KM>;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
    return REAXMOE_ERR_CUDA;
  kfn<<<grid, THREADS, SMEM_BYTES, s>>>(prm);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : REAXMOE_ERR_CUDA;
}

}  // namespace router

int launch_router_topk(const RouterLaunch& r, cudaStream_t s) {
  using namespace router;
  if (r.T == 0) return 0;
  Params prm;
  memset(&prm, 0, sizeof(prm));
  if (sm100::make_map(&prm.tmX, r.x, r.T, r.H * 2, BM)) return REAXMOE_ERR_CUDA;
  if (sm100::make_map(&prm.tmW, r.w, r.E, r.H * 2, r.E)) return REAXMOE_ERR_CUDA;
  prm.scale = static_cast<const __nv_bfloat16*>(r.scale);
  prm.pes = r.pes;
  prm.root = r.root;
  prm.eps = r.eps;
  prm.T = r.T;
  prm.H = r.H;
  prm.E = r.E;
  prm.K = r.K;
  prm.ids = r.ids;
  prm.wts = r.wts;
  prm.logits = r.logits;
  prm.status = r.status;
  prm.timeout_ns = r.timeout_ns;
  const int64_t tiles = ceil_div64(r.T, BM);
  const int grid = (int)(tiles < r.num_sms ? tiles : r.num_sms);   // persistent: at most one CTA per SM
  const bool k8 = r.K <= 8;
  switch (r.E) {
    case 32: return k8 ? launch_e<32, 8>(prm, grid, s) : launch_e<32, 16>(prm, grid, s);
    case 64: return k8 ? launch_e<64, 8>(prm, grid, s) : launch_e<64, 16>(prm, grid, s);
    case 128: return k8 ? launch_e<128, 8>(prm, grid, s) : launch_e<128, 16>(prm, grid, s);
    default: return REAXMOE_ERR_UNSUPPORTED;
  }
}

}  // namespace reaxmoe
