// gemm_sm100.cu -- persistent grouped NVFP4 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces the reference's sm_120a grouped GEMMs (champions/uid240/opt/blink/blink_moegemm.cu:472-934 "bmoe"
// MODE 0/1 and bmoe69.cu variant 11) and the stock vLLM cutlass_fp4_moe_mm + activation + quant chain
// (vllm/model_executor/layers/fused_moe/experts/cutlass_moe.py:609-648). Same arithmetic per output element:
//   acc = sum over K of e2m1(A) * e4m3(sfA) * e2m1(B) * e4m3(sfB)   (block-scaled MMA, fp32 accumulation)
//   mode 0 (w2):  out = bf16(alpha_e * acc)
//   mode 1 (w13): gate/up = bf16(alpha_e * acc); h = bf16(bf16(act(gate)) * up); NVFP4 quant of h with the
//                 expert's intermediate scale (engine/fp4.py numerics) -> FP4 rows + 128x4 scale atoms.
//
// Design (one CTA per SM, persistent). Work is handed out round-robin over the CTAs: one m-tile (expert, 128 routed
// rows) with all its n-tiles (256 output columns each; a narrower last n-tile of 128 when N % 256 == 128) per item,
// in full waves of one m-tile per CTA; the m-tiles left after the last full wave go out as single (m-tile, n-tile)
// units, so that the kernel's tail is a fraction of an m-tile on every CTA instead of a whole m-tile on some. A small
// batch (fewer than two m-tiles per CTA) is all units, so that every SM takes part in reading the weights (measured
// at 1024 skewed tokens: 0.378 -> 0.215 ms per layer).
//   warp 0      TMA producer, into a 4-deep ring of 54 KiB stages: A (routed FP4 rows, 128 x 256 K) and B (expert
//               weights, 256 x 256 K) by 2D TMA with 128-byte swizzle, plus the stage's scale atoms as they lie in
//               memory (engine/fp4.py 128x4 atoms, 512 B per 128 rows x 64-element k-chunk) by 1D bulk copies: the
//               A scales of the m-tile's rows and the B scales of the n-tile's two 128-row blocks. Resident-A layout
//               (K <= 768, i.e. w2, with at least two m-tiles per CTA): the m-tile's whole A and its scale atoms
//               (up to 3 slices of 256 K, 54 KiB) are loaded once per m-tile into a fixed region and read by all its
//               n-tiles, and the ring stages (36 KiB) carry B and its scale atoms only. Each slice has its own
//               full / empty barrier pair: the next m-tile's slice is loaded as soon as the last n-tile's MMAs on it
//               are done (measured at config 2: w2 0.567 -> 0.548 ms).
//   warps 2-3   gather layout (w13 when every expert quantises its input with the same scale): the A tile of each
//               stage by 16-byte cp.async from token-major FP4 rows through the slot -> token map, written in the
//               128-byte-swizzled layout a TMA box gives, then one cp.async arrive per thread on the stage's full
//               barrier. The routed rows are then never replicated in HBM (the reference's gather-A variant,
//               blink_moegemm.cu:532-647, reads its A rows through a_map the same way). Idle otherwise.
//   warp 1      allocates 512 TMEM columns; one thread issues tcgen05.mma.kind::mxf4nvf4.block_scale.block16
//               (M=128, N=256, K=64; 4 per stage) into the fp32 accumulator and commits each stage to its empty
//               barrier (which frees the stage's shared memory and its scale columns in TMEM).
//   warps 4-7   scale writers, one per TMEM lane quarter: each lane reads one 16-byte row of every scale atom of the
//               stage from shared memory and writes it into its lane with tcgen05.st -- the TMEM image the MMA reads
//               (A: lane i gets atom row i in 4 columns; B: atom row i of block 0 then of block 1 in 8 columns,
//               replicated in every quarter). Written from registers, these stores do not queue in the tensor pipe
//               behind the running MMAs (a tcgen05.cp would, and the next stage's MMAs would wait on its commit).
//   warps 8-15  epilogue: tcgen05.ld the whole accumulator into registers (each warp owns its 32-lane TMEM quarter and
//               half of the columns) and release it to the MMA warp at once,
//               then convert / activate / quantise and store while the next unit's MMAs run.
// TMEM: accumulator [0, 256); per stage, A scales (16 columns) and B scales (32 columns) -- 448 columns in all.
// Every mbarrier wait is bounded (globaltimer); on expiry the CTA records REAXMOE_ERR_DEVICE_TIMEOUT in the
// status word, raises a CTA-wide abort flag, drains its own in-flight copies and MMAs, frees TMEM and returns.
// Plain per-CTA TMA loads, no thread-block clusters: the same kernel runs on every rank of the expert-parallel path.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

namespace reaxmoe {
namespace gemm {

using namespace sm100;

constexpr int BM = 128;                 // rows per tile (MMA M)
constexpr int BN = 256;                 // cols per tile (MMA N); mode 1: 128 gate + 128 up columns
constexpr int KSTEP = 64;               // K per tcgen05.mma (FP4)
constexpr int KSTAGE = 256;             // K per pipeline stage = one 128-byte swizzle row of FP4
constexpr int KPS = KSTAGE / KSTEP;     // MMAs per stage
constexpr int A_BYTES = BM * KSTAGE / 2;
constexpr int B_BYTES = BN * KSTAGE / 2;
constexpr int SF_ATOM = 512;            // scales of 128 rows x one 64-element k-chunk (a 128x4 atom)
constexpr int SFA_BYTES = KPS * SF_ATOM;        // the stage's A scale atoms
constexpr int SFB_BYTES = 2 * KPS * SF_ATOM;    // the stage's B scale atoms: block 0 (rows 0-127), then block 1
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
constexpr int STAGES = 4;
// Four warpgroups: 0 = producer (warp 0), MMA issuer (warp 1), two idle warps; 1 = the scale writers (warps 4-7, one
// per TMEM lane quarter); 2 and 3 = the epilogue (warps 8-15, two per lane quarter, each half of the tile's columns).
// Launched with 128 registers a thread; warpgroups 0 and 1 hand registers to the epilogue with setmaxnreg
// (2 x 128 x 56 + 2 x 128 x 200 = 65536, the launch's total).
constexpr int SCALE_WARP0 = 4;
constexpr int GA_WARP0 = 2;             // gather layout: warps 2-3 fetch the A rows by cp.async
constexpr int GA_THREADS = 64;
constexpr int EPI_WARP0 = 8;
constexpr int NUM_EPI_WARPS = 8;
constexpr int THREADS = (EPI_WARP0 + NUM_EPI_WARPS) * 32;
constexpr int REGS_CONTROL = 56;
constexpr int REGS_EPILOGUE = 200;
static_assert(2 * 128 * REGS_CONTROL + 2 * 128 * REGS_EPILOGUE <= 65536, "register split above the launch total");
constexpr int TMEM_COLS = 512;
constexpr int SFA_COL = BN;                           // A scales of stage s: columns SFA_COL + 16 s + 4 kk
constexpr int SFB_COL = SFA_COL + STAGES * 4 * KPS;   // B scales of stage s: columns SFB_COL + 32 s + 8 kk
// Resident A (problems with K <= 768, i.e. w2 at the 26B-A4B shapes): the m-tile's whole A -- at most RA_SLICES
// slices of 256 K -- and its scale atoms are loaded once per work item into a fixed region and read by all the item's
// n-tiles; the ring then carries B and its scale atoms only (36 instead of 54 KiB a stage).
constexpr int RA_SLICES = 3;
constexpr int RA_BYTES = RA_SLICES * (A_BYTES + SFA_BYTES);
constexpr int NUM_BARS = 3 * STAGES + 3 + 2 * RA_SLICES;
constexpr int GA_ROWS_INTS = 128;        // gather layout: the current item's 128 A source rows
constexpr int SMEM_TABLE_INTS = 4 * (kMaxExperts + 1) + GA_ROWS_INTS;
template <bool RA>
struct Layout {
  static constexpr int stage = RA ? B_BYTES + SFB_BYTES : STAGE_BYTES;  // bytes of one ring stage
  static constexpr int ring = RA ? RA_BYTES : 0;                        // offset of stage 0
  static constexpr int b_off = RA ? 0 : A_BYTES;                        // B tile inside a stage
  static constexpr int sfb_off = RA ? B_BYTES : A_BYTES + B_BYTES + SFA_BYTES;
  static constexpr int bars = ring + STAGES * stage;
  static constexpr int smem = 1024 + bars + 256 + SMEM_TABLE_INTS * 4;
  static_assert(stage % 1024 == 0 && ring % 1024 == 0, "tiles must stay 1024-byte aligned for the 128B swizzle");
  static_assert(smem <= 227 * 1024, "shared memory budget");
};
static_assert(SFB_COL + STAGES * 8 * KPS <= TMEM_COLS, "TMEM budget");
static_assert(NUM_BARS * 8 + 8 <= 256, "barrier area");

// Instruction descriptor of tcgen05.mma.kind::mxf4nvf4 (block-scaled): A/B = e2m1 (MXF4 format 1) at bits
// [7,10) / [10,13), K-major both, N >> 3 at [17,23), scale type ue4m3 (0) at bit 23, M >> 4 at [24,29),
// scale-factor ids 0, dense K = 64.
__host__ __device__ constexpr uint32_t idesc_for(int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

struct Params {
  CUtensorMap tmA;  // [slots, K/2] u8, box 128 bytes x 128 rows, 128B swizzle
  CUtensorMap tmB;  // [E*N, K/2] u8, box 128 bytes x 256 rows, 128B swizzle
  const uint8_t* sfA;   // A scale atoms [row blocks][k_chunks][512] (blockscale_offsets rows)
  const uint8_t* sfB;   // B scale atoms as engine/fp4.py lays them out: [E][N/128][k_chunks][512]
  const float* alphas;
  const int* counts;
  const int* eoff;
  const int* boff;
  const int* tile_prefix;
  __nv_bfloat16* out;
  uint8_t* q_out;
  uint8_t* q_sf;
  const float* q_gscale;
  int* status;
  unsigned long long timeout_ns;
  const uint64_t* direct_dst;  // mode 0: per slot row, its record's return address (0 = write c3)
  const float* direct_w;
  // gather layout (mode 1): A rows from ga_tok [ga_tokens, K/2] through row_token when *ga_flag is set, else from the
  // per-slot rows ga_rep [slots, K/2]
  const uint8_t* ga_tok;
  const uint8_t* ga_rep;
  const int* row_token;
  const int* ga_flag;
  int64_t ga_tokens;
  int64_t ga_stride;    // bytes between consecutive gathered rows (K/2, or the expert-parallel record size)
  int64_t slots;
  int topk;
  int E, N, K, n_tiles, k_chunks, n_blocks;
  int tail_n;           // width of the last n-tile (256, or 128 when N % 256 == 128)
};

__device__ __forceinline__ void tc_mma_fp4(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                           uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

struct MTile {
  int e, mt, row0, rows, sfblk;
};

// m-tile gm (global index over all experts' 128-row tiles) -> expert, tile inside the expert, first routed row,
// valid rows and its scale-atom row block.
__device__ __forceinline__ MTile decode_mtile(int gm, int E, const int* s_tp, const int* s_cnt, const int* s_eoff,
                                              const int* s_boff) {
  int lo = 0, hi = E;  // largest e < E with s_tp[e] <= gm
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_tp[mid] <= gm) lo = mid; else hi = mid;
  }
  MTile r;
  r.e = lo;
  r.mt = gm - s_tp[lo];
  r.row0 = s_eoff[lo] + r.mt * BM;
  r.rows = min(BM, s_cnt[lo] - r.mt * BM);
  r.sfblk = (s_boff[lo] >> 7) + r.mt;
  return r;
}

// Two fp32 lanes in one 64-bit register, for Blackwell's packed fp32x2 instructions (each lane rounds exactly as
// the scalar instruction would).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// the hardware base-2 exponential and reciprocal approximations (ex2.approx, rcp.approx; about 2^-22 relative)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 1 / (1 + 2^z) on both lanes
__device__ __forceinline__ uint64_t f2_rcp_one_plus_ex2(uint64_t z) {
  float zl, zh, dl, dh;
  f2_unpack(z, zl, zh);
  f2_unpack(f2_add(f2_pack(ex2_approx(zl), ex2_approx(zh)), f2_pack(1.0f, 1.0f)), dl, dh);
  return f2_pack(rcp_approx(dl), rcp_approx(dh));
}
// The gate activation on two lanes, from the definitions:
//   GELU with the tanh approximation (blink_moegemm.cu:349-355): 0.5 x (1 + tanh(y)), y = sqrt(2/pi) (x + 0.044715 x^3).
//     With tanh(y) = 1 - 2 r, r = 1 / (1 + e^(2y)): 0.5 x (1 + tanh(y)) = x - x r, and e^(2y) = 2^z with
//     z = x (C + 0.044715 C x^2), C = 2 sqrt(2/pi) log2(e). Saturates to x (r = 0) and to 0 (r = 1).
//   SiLU: x / (1 + e^(-x)) = x r, r = 1 / (1 + 2^(-x log2(e))).
template <int ACT>
__device__ __forceinline__ uint64_t act2(uint64_t x) {
  if constexpr (ACT == REAXMOE_ACT_GELU_TANH) {
    constexpr float kC = 2.302208185195923f;       // 2 sqrt(2/pi) log2(e)
    constexpr float kKC = 0.10294324159622192f;    // 0.044715 C
    const uint64_t z = f2_mul(x, f2_fma(f2_pack(kKC, kKC), f2_mul(x, x), f2_pack(kC, kC)));
    return f2_fma(x ^ 0x8000000080000000ull, f2_rcp_one_plus_ex2(z), x);
  } else {
    constexpr float kNL = -1.4426950216293335f;    // -log2(e)
    return f2_mul(x, f2_rcp_one_plus_ex2(f2_mul(x, f2_pack(kNL, kNL))));
  }
}

// Fused w13 epilogue for one thread: 32 gate and 32 up accumulators of one row -> 16 packed FP4 bytes + 2 scale
// bytes. gate/up = bf16(alpha * acc); h = bf16(bf16(act(gate)) * up) (a bf16 product of two bf16 values rounds
// exactly like the fp32 product rounded to bf16); NVFP4 quantisation of h with engine/fp4.py numerics, by the bf16x2
// quantiser (h is exactly bf16). The fp32 work runs on lane pairs (fp32x2 instructions).
template <int ACT>
__device__ __forceinline__ uint32_t act_quant32(const uint32_t (&x0)[32], const uint32_t (&x1)[32], float alpha,
                                                float g, uint32_t (&w)[4]) {
  const uint64_t al = f2_pack(alpha, alpha);
  uint32_t sbytes = 0u;
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    uint32_t hw[8];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      float gl, gh, ul, uh, al_, ah;
      f2_unpack(f2_mul(f2_pack(__uint_as_float(x0[16 * b + i]), __uint_as_float(x0[16 * b + i + 1])), al), gl, gh);
      f2_unpack(f2_mul(f2_pack(__uint_as_float(x1[16 * b + i]), __uint_as_float(x1[16 * b + i + 1])), al), ul, uh);
      const __nv_bfloat162 gb = __floats2bfloat162_rn(gl, gh);
      const __nv_bfloat162 ub = __floats2bfloat162_rn(ul, uh);
      const float2 gf = __bfloat1622float2(gb);
      f2_unpack(act2<ACT>(f2_pack(gf.x, gf.y)), al_, ah);
      const __nv_bfloat162 ab = __floats2bfloat162_rn(al_, ah);
      const __nv_bfloat162 h2 = __hmul2(ab, ub);
      hw[i / 2] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    sbytes |= quant_block16_bf16(hw, g, w[2 * b], w[2 * b + 1]) << (8 * b);
  }
  return sbytes;
}

template <int MODE, int ACT, bool RA, bool GA>
__global__ void __launch_bounds__(THREADS, 1) grouped_gemm_kernel(const __grid_constant__ Params p) {
  static_assert(!(GA && RA), "the gather layout uses the ring for A");
  using L = Layout<RA>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem + L::ring;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* full = bars;                 // [STAGES] A, B and the scale atoms landed (TMA tx)
  uint64_t* empty = bars + STAGES;       // [STAGES] MMAs of the stage done: smem stage and its TMEM scales free
  uint64_t* sff = empty + STAGES;        // [STAGES] the stage's scales written to TMEM (4 scale-writer warps)
  uint64_t* accf = sff + STAGES;         // accumulator ready for the epilogue
  uint64_t* acce = accf + 1;             // accumulator drained by the epilogue
  uint64_t* drain_mma = acce + 1;
  uint64_t* afull = drain_mma + 1;       // [RA_SLICES] resident A slice and its scale atoms landed
  uint64_t* aempty = afull + RA_SLICES;  // [RA_SLICES] the item's last MMAs on the slice done: slice free
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(aempty + RA_SLICES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  int* s_tp = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(bars) + 256);
  int* s_cnt = s_tp + (kMaxExperts + 1);
  int* s_eoff = s_cnt + (kMaxExperts + 1);
  int* s_boff = s_eoff + (kMaxExperts + 1);
  uint32_t* s_garows = reinterpret_cast<uint32_t*>(s_boff + (kMaxExperts + 1));   // [8 r0][16 i]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int E = p.E;
  for (int i = threadIdx.x; i <= E; i += blockDim.x) {
    s_tp[i] = p.tile_prefix[i];
    if (i < E) {
      s_cnt[i] = p.counts[i];
      s_eoff[i] = p.eoff[i];
      s_boff[i] = p.boff[i];
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      // gather layout: the producer's expect-tx arrive plus one cp.async arrive per gathering thread
      mbar_init(smem_u32(&full[s]), GA ? 1 + GA_THREADS : 1);
      mbar_init(smem_u32(&empty[s]), 1);
      mbar_init(smem_u32(&sff[s]), 4);
    }
    mbar_init(smem_u32(accf), 1);
    mbar_init(smem_u32(acce), NUM_EPI_WARPS);
    mbar_init(smem_u32(drain_mma), 1);
    for (int s = 0; s < RA_SLICES; ++s) {
      mbar_init(smem_u32(&afull[s]), 1);
      mbar_init(smem_u32(&aempty[s]), 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tmB)) : "memory");
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
  const int n_tiles = p.n_tiles;
  const int total_mtiles = s_tp[E];
  // Work items, handed out round-robin (so that the CTAs in flight share a few experts' weights in L2): whole
  // m-tiles with all their n-tiles in full waves of gridDim.x, then the remaining m-tiles as single (m-tile, n-tile)
  // units spread over all CTAs, so that no CTA runs a whole extra m-tile while the others idle. A small batch (fewer
  // than two m-tiles per CTA) is all units, so that every SM takes part in the weight reads.
  const int whole = total_mtiles < 2 * (int)gridDim.x ? 0 : total_mtiles / (int)gridDim.x * (int)gridDim.x;
  const int items = whole + (total_mtiles - whole) * n_tiles;
  auto item_mtile = [&](int u) { return u < whole ? u : whole + (u - whole) / n_tiles; };
  auto item_nt0 = [&](int u) { return u < whole ? 0 : (u - whole) % n_tiles; };
  auto item_nts = [&](int u) { return u < whole ? n_tiles : 1; };
  const int k_chunks = p.k_chunks;
  const int k_stages = (k_chunks + KPS - 1) / KPS;
  // the n-tile's second 128-row block of B exists unless it is the narrow last tile
  auto has_block1 = [&](int nt) { return nt < n_tiles - 1 || p.tail_n == BN; };
  if (warp < EPI_WARP0) {
    // warpgroups 0 and 1: producer, MMA issuer, scale writers (two idle warps); their registers go to the epilogue
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CONTROL));
    if (warp == 0) {
      // ------------------------------------------------------------------ TMA producer
      if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        long fills = 0;
        int a_fills[RA_SLICES] = {0, 0, 0};
        bool ok = true;
        for (int u = blockIdx.x, it = 0; u < items && ok; u += gridDim.x, ++it) {
          const MTile M = decode_mtile(item_mtile(u), E, s_tp, s_cnt, s_eoff, s_boff);
          const uint8_t* sfa = p.sfA + (size_t)M.sfblk * k_chunks * SF_ATOM;
          const int nt_first = item_nt0(u);
          for (int nt = nt_first, nt_end = nt + item_nts(u); nt < nt_end && ok; ++nt) {
            const int brow = M.e * p.N + nt * BN;
            const bool b1 = has_block1(nt);
            const uint8_t* sfb0 = p.sfB + ((size_t)M.e * p.n_blocks + 2 * nt) * k_chunks * SF_ATOM;
            const uint8_t* sfb1 = sfb0 + (size_t)k_chunks * SF_ATOM;
            for (int ks = 0; ks < k_stages; ++ks) {
              const int kc0 = ks * KPS;
              const int nk = min(KPS, k_chunks - kc0);
              const uint32_t sf_bytes = (uint32_t)(nk * SF_ATOM);
              if (RA && nt == nt_first) {
                // the item's A slice ks, once the previous item's MMAs on it are done
                if (!wait_bounded(smem_u32(&aempty[ks]), (uint32_t)(it & 1) ^ 1u, abort_flag, p.status,
                                  p.timeout_ns)) {
                  ok = false;
                  break;
                }
                const uint32_t abar = smem_u32(&afull[ks]);
                mbar_expect_tx(abar, (uint32_t)A_BYTES + sf_bytes);
                tma_load_2d(smem_u32(smem + ks * A_BYTES), &p.tmA, abar, kc0 * (KSTEP / 2), M.row0);
                bulk_load(smem_u32(smem + RA_SLICES * A_BYTES + ks * SFA_BYTES), sfa + (size_t)kc0 * SF_ATOM,
                          sf_bytes, abar);
                ++a_fills[ks];
              }
              if (!wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.status, p.timeout_ns)) {
                ok = false;
                break;
              }
              uint8_t* st = ring + stage * L::stage;
              const uint32_t bar = smem_u32(&full[stage]);
              uint8_t* sfb_st = st + L::sfb_off;
              if constexpr (RA) {
                mbar_expect_tx(bar, (uint32_t)B_BYTES + sf_bytes * (b1 ? 2u : 1u));
              } else if constexpr (GA) {
                // the A tile comes from the gathering warps
                mbar_expect_tx(bar, (uint32_t)B_BYTES + sf_bytes * (b1 ? 3u : 2u));
                bulk_load(smem_u32(st + A_BYTES + B_BYTES), sfa + (size_t)kc0 * SF_ATOM, sf_bytes, bar);
              } else {
                mbar_expect_tx(bar, (uint32_t)(A_BYTES + B_BYTES) + sf_bytes * (b1 ? 3u : 2u));
                tma_load_2d(smem_u32(st), &p.tmA, bar, kc0 * (KSTEP / 2), M.row0);
                bulk_load(smem_u32(st + A_BYTES + B_BYTES), sfa + (size_t)kc0 * SF_ATOM, sf_bytes, bar);
              }
              tma_load_2d(smem_u32(st + L::b_off), &p.tmB, bar, kc0 * (KSTEP / 2), brow);
              bulk_load(smem_u32(sfb_st), sfb0 + (size_t)kc0 * SF_ATOM, sf_bytes, bar);
              if (b1) bulk_load(smem_u32(sfb_st + KPS * SF_ATOM), sfb1 + (size_t)kc0 * SF_ATOM, sf_bytes, bar);
              ++fills;
              if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
          }
        }
        // let the last fills land before the CTA may exit (only matters after an abort)
        for (long f = fills - 1; f >= 0 && f >= fills - STAGES; --f)
          wait_drain(smem_u32(&full[f % STAGES]), (uint32_t)((f / STAGES) & 1));
        if constexpr (RA) {
          for (int ks = 0; ks < RA_SLICES; ++ks)
            if (a_fills[ks] > 0) wait_drain(smem_u32(&afull[ks]), (uint32_t)((a_fills[ks] - 1) & 1));
        }
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------------ MMA issuer (one thread)
      if (lane == 0) {
        long n = 0;  // global stage counter of this CTA
        uint32_t acc_phase = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < items && ok; u += gridDim.x) {
          for (int nt = item_nt0(u), nt_end = nt + item_nts(u); nt < nt_end && ok; ++nt) {
            const uint32_t idesc = idesc_for(nt == n_tiles - 1 ? p.tail_n : BN);
            if (!wait_bounded(smem_u32(acce), acc_phase ^ 1u, abort_flag, p.status, p.timeout_ns)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int ks = 0; ks < k_stages; ++ks, ++n) {
              const int stage = (int)(n % STAGES);
              const int nk = min(KPS, k_chunks - ks * KPS);
              // the stage's scales are in TMEM (the writers waited for the stage's TMA data first, so the A/B tiles
              // have landed as well)
              if (!wait_bounded(smem_u32(&sff[stage]), (uint32_t)((n / STAGES) & 1), abort_flag, p.status,
                                p.timeout_ns)) {
                ok = false;
                break;
              }
              tc_fence_after();
              if constexpr (GA) fence_proxy_async_smem();   // A was written by cp.async (generic proxy)
              const uint32_t st = smem_u32(ring + stage * L::stage);
              const uint32_t a_s = RA ? smem_u32(smem + ks * A_BYTES) : st;
              const uint32_t b_s = st + L::b_off;
              for (int kk = 0; kk < nk; ++kk)
                tc_mma_fp4(tmem, desc_sw128(a_s + kk * (KSTEP / 2)), desc_sw128(b_s + kk * (KSTEP / 2)), idesc,
                           tmem + SFA_COL + 4 * (KPS * stage + kk), tmem + SFB_COL + 8 * (KPS * stage + kk),
                           (ks | kk) != 0 ? 1u : 0u);
              tc_commit(smem_u32(&empty[stage]));
              // the item's last MMAs on the resident slice: it may be refilled once they complete
              if (RA && nt == nt_end - 1) tc_commit(smem_u32(&aempty[ks]));
            }
            if (!ok) break;
            tc_commit(smem_u32(accf));
            acc_phase ^= 1u;
          }
        }
        // all tcgen05 work of this thread has completed once this commit arrives
        tc_commit(smem_u32(drain_mma));
        wait_drain(smem_u32(drain_mma), 0);
      }
    } else if (GA && warp >= GA_WARP0 && warp < GA_WARP0 + GA_THREADS / 32) {
      // ------------------------------------------------------------------ A gather (gather layout, warps 2-3)
      // Each stage's A tile, 128 rows x 128 bytes, by 16-byte cp.async into the 128-byte-swizzled layout a TMA load
      // would give (16-byte piece c of row r at r * 128 + (c ^ (r % 8)) * 16). Thread g takes piece g % 8 of rows
      // g / 8 + 8 i: one warp instruction reads four whole 128-byte row slices. The item's source rows are looked up
      // once per work item into a shared table ([g / 8][i], filled by the eight lanes that share g / 8, in their
      // own warp) and read back per stage. A row past the m-tile's routed rows repeats its first row (the epilogue
      // drops it); source rows are clamped to the array.
      constexpr int RPT = BM / 8;                                // rows per thread
      const int g = threadIdx.x - GA_WARP0 * 32;
      const int piece = g & 7, r0 = g >> 3;
      const bool from_tok = *p.ga_flag != 0;
      const uint8_t* base = from_tok ? p.ga_tok : p.ga_rep;
      const int64_t nrows = from_tok ? p.ga_tokens : p.slots;
      const uint32_t rb = (uint32_t)(from_tok ? p.ga_stride : p.K / 2);
      const uint32_t dpiece = (uint32_t)((piece ^ r0) << 4);   // r % 8 == r0 for every row of this thread
      uint32_t* rows_tab = s_garows + r0 * RPT;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < items && ok; u += gridDim.x) {
        const MTile M = decode_mtile(item_mtile(u), E, s_tp, s_cnt, s_eoff, s_boff);
        __syncwarp();   // the previous item's table reads are done
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int i = 2 * piece + j;
          const int r = r0 + 8 * i;
          const int64_t slot = (int64_t)M.row0 + (r < M.rows ? r : 0);
          const int64_t v = from_tok ? (int64_t)__ldg(p.row_token + slot) : slot;
          rows_tab[i] = (uint32_t)(v < 0 ? 0 : (v >= nrows ? nrows - 1 : v));
        }
        __syncwarp();
        for (int nt = item_nt0(u), nt_end = nt + item_nts(u); nt < nt_end && ok; ++nt) {
          for (int ks = 0; ks < k_stages; ++ks) {
            const int kc0 = ks * KPS;
            const int nk = min(KPS, k_chunks - kc0);
            bool free_slot = false;
            if (lane == 0)
              free_slot = wait_bounded(smem_u32(&empty[stage]), phase ^ 1u, abort_flag, p.status, p.timeout_ns);
            if (__shfl_sync(0xffffffffu, free_slot ? 1 : 0, 0) == 0) {
              ok = false;
              break;
            }
            const uint32_t st = smem_u32(ring + stage * L::stage) + (uint32_t)(r0 * 128) + dpiece;
            if (piece < 2 * nk) {
              const uint8_t* col = base + kc0 * (KSTEP / 2) + piece * 16;
#pragma unroll
              for (int q = 0; q < RPT / 4; ++q) {
                const uint4 sr = *reinterpret_cast<const uint4*>(rows_tab + 4 * q);
                cp_async_16(st + (uint32_t)((4 * q + 0) * 8 * 128), col + (uint64_t)sr.x * rb);
                cp_async_16(st + (uint32_t)((4 * q + 1) * 8 * 128), col + (uint64_t)sr.y * rb);
                cp_async_16(st + (uint32_t)((4 * q + 2) * 8 * 128), col + (uint64_t)sr.z * rb);
                cp_async_16(st + (uint32_t)((4 * q + 3) * 8 * 128), col + (uint64_t)sr.w * rb);
              }
            }
            cp_async_arrive_noinc(smem_u32(&full[stage]));
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      cp_async_wait_all();
    } else if (warp >= SCALE_WARP0 && warp < EPI_WARP0) {
      // ------------------------------------------------------------------ scale writers (one warp per lane quarter)
      // A stage's TMEM scale columns are free once its previous MMAs completed; the producer waited for that (the
      // stage's empty barrier) before refilling the stage, so the stage's full barrier implies it.
      const uint32_t tq = tmem + ((uint32_t)((warp & 3) * 32) << 16);
      long n = 0;
      bool ok = true;
      const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
      for (int u = blockIdx.x, it = 0; u < items && ok; u += gridDim.x, ++it) {
        const int nt_first = item_nt0(u);
        for (int nt = nt_first, nt_end = nt + item_nts(u); nt < nt_end && ok; ++nt) {
          const bool b1 = has_block1(nt);
          for (int ks = 0; ks < k_stages; ++ks, ++n) {
            const int stage = (int)(n % STAGES);
            const int nk = min(KPS, k_chunks - ks * KPS);
            // one lane waits, the warp follows its verdict (the stores below are warp-collective); with a resident
            // A, the item's first n-tile also waits for the A slice (its scale atoms are read below, and the MMA
            // issuer, which waits for this warp's arrival, reads the slice)
            bool landed = false;
            if (lane == 0) {
              landed = !(RA && nt == nt_first) ||
                       wait_bounded(smem_u32(&afull[ks]), (uint32_t)(it & 1), abort_flag, p.status, p.timeout_ns);
              landed = landed && wait_bounded(smem_u32(&full[stage]), (uint32_t)((n / STAGES) & 1), abort_flag,
                                              p.status, p.timeout_ns);
            }
            landed = __shfl_sync(0xffffffffu, landed ? 1 : 0, 0) != 0;
            if (!landed) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint8_t* sfa_st = (RA ? smem + RA_SLICES * A_BYTES + ks * SFA_BYTES
                                        : ring + stage * L::stage + A_BYTES + B_BYTES) + lane * 16;
            const uint8_t* sfb_st = ring + stage * L::stage + L::sfb_off + lane * 16;
            for (int kk = 0; kk < nk; ++kk) {
              const uint4 a = *reinterpret_cast<const uint4*>(sfa_st + kk * SF_ATOM);
              const uint4 b0 = *reinterpret_cast<const uint4*>(sfb_st + kk * SF_ATOM);
              const uint4 bb = b1 ? *reinterpret_cast<const uint4*>(sfb_st + (KPS + kk) * SF_ATOM) : zero;
              tc_st_32x32b_x4(tq + SFA_COL + 4 * (KPS * stage + kk), a);
              tc_st_32x32b_x8(tq + SFB_COL + 8 * (KPS * stage + kk), b0, bb);
            }
            tc_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&sff[stage]));
          }
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_EPILOGUE));
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;                       // TMEM lane quarter this warp may access
    const int sub = (warp - EPI_WARP0) >> 2;      // which half of the tile's columns
    const int r = q * 32 + lane;                  // row inside the tile
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < items && ok; u += gridDim.x) {
      const MTile M = decode_mtile(item_mtile(u), E, s_tp, s_cnt, s_eoff, s_boff);
      const int64_t row = (int64_t)M.row0 + r;
      // expert-parallel receiver: a slot that is its record's only local pair is written as the finished row
      uint64_t direct = 0ull;
      float wdir = 0.0f;
      if constexpr (MODE == 0) {
        if (p.direct_dst != nullptr && r < M.rows) {
          direct = p.direct_dst[row];
          wdir = bf16r(p.direct_w[row]);
        }
      }
      for (int nt = item_nt0(u), nt_end = nt + item_nts(u); nt < nt_end; ++nt) {
        const int un = (nt == n_tiles - 1) ? p.tail_n : BN;
        if (!wait_bounded(smem_u32(accf), acc_phase, abort_flag, p.status, p.timeout_ns)) {
          ok = false;
          break;
        }
        acc_phase ^= 1u;
        tc_fence_after();
        const uint32_t t_base = tmem + ((uint32_t)(q * 32) << 16);
        // full tiles: this warp's 128 output columns (mode 0) or 64 gate + 64 up columns (mode 1);
        // the narrow last tile: 64 columns (mode 0) or 32 gate + 32 up (mode 1)
        const int half = un / 2;
        uint32_t x[4][32];
        if constexpr (MODE == 0) {
          // this warp's half = 128 columns (64 in the narrow last tile)
          const int cw = un / 2;
          tc_ld_32x32b_x32(t_base + sub * cw, x[0]);
          tc_ld_32x32b_x32(t_base + sub * cw + 32, x[1]);
          if (un == BN) {
            tc_ld_32x32b_x32(t_base + sub * cw + 64, x[2]);
            tc_ld_32x32b_x32(t_base + sub * cw + 96, x[3]);
          }
        } else {
          const int hw = un / 4;                  // h columns per warp half
          tc_ld_32x32b_x32(t_base + sub * hw, x[0]);             // gate
          tc_ld_32x32b_x32(t_base + half + sub * hw, x[1]);      // up
          if (un == BN) {
            tc_ld_32x32b_x32(t_base + sub * hw + 32, x[2]);
            tc_ld_32x32b_x32(t_base + half + sub * hw + 32, x[3]);
          }
        }
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(acce));
        if (r >= M.rows) continue;
        const float alpha = p.alphas[M.e];
        if constexpr (MODE == 0) {
          // 32 columns per x[j] -> 64 bytes of bf16 -> two full 32-byte sectors per 256-bit store
          const int col0 = nt * BN + sub * (un / 2);
          uint8_t* dst = direct != 0ull ? reinterpret_cast<uint8_t*>(direct) + (size_t)col0 * 2
                                        : reinterpret_cast<uint8_t*>(p.out + row * p.N + col0);
          const int nq = un == BN ? 4 : 2;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (j < nq) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint32_t o[8];
                if (direct != 0ull) {
                  // the combine of a record with one pair: bf16(bf16(c3) * bf16(w)); its fp32 sum with the
                  // absent pairs' +0 terms turns -0 into +0 when topk > 1
#pragma unroll
                  for (int i = 0; i < 8; ++i) {
                    float v0 = bf16r(__fmul_rn(bf16r(alpha * __uint_as_float(x[j][16 * h + 2 * i])), wdir));
                    float v1 = bf16r(__fmul_rn(bf16r(alpha * __uint_as_float(x[j][16 * h + 2 * i + 1])), wdir));
                    if (p.topk > 1) {
                      v0 = __fadd_rn(v0, 0.0f);
                      v1 = __fadd_rn(v1, 0.0f);
                    }
                    o[i] = pack_bf16x2(v0, v1);
                  }
                } else {
#pragma unroll
                  for (int i = 0; i < 8; ++i)
                    o[i] = pack_bf16x2(alpha * __uint_as_float(x[j][16 * h + 2 * i]),
                                       alpha * __uint_as_float(x[j][16 * h + 2 * i + 1]));
                }
                st_global_v8(dst + 64 * j + 32 * h, o);
              }
            }
          }
        } else {
          const int inter = p.N / 2;
          const float g = __fdiv_rn(1.0f, p.q_gscale[M.e]);
          const int hw = un / 4;
          const int c0 = nt * (BN / 2) + sub * hw;   // first intermediate column of this thread's slice
          uint8_t* qrow = p.q_out + row * (inter / 2);
          const int64_t sfrow = (int64_t)M.sfblk * 128 + r;
          uint32_t w[4];
          uint32_t sb = act_quant32<ACT>(x[0], x[1], alpha, g, w);
          *reinterpret_cast<uint4*>(qrow + c0 / 2) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint16_t*>(p.q_sf + sf_offset(sfrow, c0 / 16, inter / 64)) = (uint16_t)sb;
          if (un == BN) {
            sb = act_quant32<ACT>(x[2], x[3], alpha, g, w);
            *reinterpret_cast<uint4*>(qrow + c0 / 2 + 16) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint16_t*>(p.q_sf + sf_offset(sfrow, c0 / 16 + 2, inter / 64)) = (uint16_t)sb;
          }
        }
      }
    }
    // direct rows went to peers' memory: fence them at system scope for the signal that follows the layer
    if (MODE == 0 && p.direct_dst != nullptr) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- host side
template <int MODE, int ACT, bool RA, bool GA = false>
static int launch_ra(const Params& prm, int grid, cudaStream_t s) {
  auto kfn = grouped_gemm_kernel<MODE, ACT, RA, GA>;
  constexpr int smem = Layout<RA>::smem;
  if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return REAXMOE_ERR_CUDA;
  kfn<<<grid, THREADS, smem, s>>>(prm);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : REAXMOE_ERR_CUDA;
}
template <int MODE, int ACT>
static int launch_t(const Params& prm, int grid, bool ra, cudaStream_t s) {
  if (ra) return launch_ra<MODE, ACT, true>(prm, grid, s);
  return launch_ra<MODE, ACT, false>(prm, grid, s);
}
template <int ACT>
static int launch_ga(const Params& prm, int grid, cudaStream_t s) {
  return launch_ra<1, ACT, false, true>(prm, grid, s);
}

}  // namespace gemm

int launch_grouped_gemm(const GemmLaunch& g, int num_sms, cudaStream_t s) {
  using namespace gemm;
  if (g.slots == 0) return 0;
  Params prm;
  memset(&prm, 0, sizeof(prm));
  int rc = make_map(&prm.tmA, g.a, g.slots, g.K / 2, BM);
  if (rc) return rc;
  rc = make_map(&prm.tmB, g.b, (int64_t)g.E * g.N, g.K / 2, BN);
  if (rc) return rc;
  prm.sfA = static_cast<const uint8_t*>(g.a_sf);
  prm.sfB = static_cast<const uint8_t*>(g.b_sf);
  prm.alphas = g.alphas;
  prm.counts = g.counts;
  prm.eoff = g.eoff;
  prm.boff = g.boff;
  prm.tile_prefix = g.tile_prefix;
  prm.out = static_cast<__nv_bfloat16*>(g.out);
  prm.q_out = static_cast<uint8_t*>(g.q_out);
  prm.q_sf = static_cast<uint8_t*>(g.q_sf);
  prm.q_gscale = g.q_gscale;
  prm.status = g.status;
  prm.timeout_ns = g.timeout_ns;
  prm.direct_dst = g.mode == 0 ? g.direct_dst : nullptr;
  prm.direct_w = g.direct_w;
  prm.topk = g.topk;
  prm.ga_tok = static_cast<const uint8_t*>(g.a_tok);
  prm.ga_rep = static_cast<const uint8_t*>(g.a);
  prm.row_token = g.row_token;
  prm.ga_flag = g.ga_flag;
  prm.ga_tokens = g.tokens;
  prm.ga_stride = g.tok_stride > 0 ? g.tok_stride : g.K / 2;
  prm.slots = g.slots;
  prm.E = g.E;
  prm.N = g.N;
  prm.K = g.K;
  if (g.N % 128 != 0) return REAXMOE_ERR_BAD_SHAPE;
  prm.n_tiles = (g.N + BN - 1) / BN;
  prm.tail_n = g.N - (prm.n_tiles - 1) * BN;   // 256 or 128
  prm.k_chunks = g.K / KSTEP;
  prm.n_blocks = g.N / 128;
  const int64_t max_units = (g.slots / BM + g.E + 1) * prm.n_tiles;
  const int grid = (int)(max_units < num_sms ? max_units : num_sms);
  // The resident-A layout where the m-tile's A fits it and every CTA gets at least two m-tiles (then the kernel
  // hands out whole m-tiles and each resident A serves all their n-tiles). A small batch, handed out as single
  // (m-tile, n-tile) units, keeps the 4-deep ring of A and B: a resident slice would only be reused by one n-tile.
  const bool ra = (prm.k_chunks + KPS - 1) / KPS <= RA_SLICES && g.slots / BM >= 2 * (int64_t)grid;
  if (g.mode == 0) return launch_t<0, 0>(prm, grid, ra, s);
  if (g.row_token != nullptr) {
    // gather layout: A through the slot -> token map, in the ring (never resident)
    if (g.ga_flag == nullptr || g.tokens < 1 || (g.tok_stride > 0 && (g.tok_stride % 16 != 0 || g.tok_stride < g.K / 2)))
      return REAXMOE_ERR_BAD_SHAPE;
    if (g.act == REAXMOE_ACT_GELU_TANH) return launch_ga<REAXMOE_ACT_GELU_TANH>(prm, grid, s);
    return launch_ga<REAXMOE_ACT_SILU>(prm, grid, s);
  }
  if (g.act == REAXMOE_ACT_GELU_TANH) return launch_t<1, REAXMOE_ACT_GELU_TANH>(prm, grid, ra, s);
  return launch_t<1, REAXMOE_ACT_SILU>(prm, grid, ra, s);
}

}  // namespace reaxmoe
