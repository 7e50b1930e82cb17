// kernels.cu -- routing, routing data, permute+quantise, combine, NVFP4 quantisation and w13 prepack kernels.
//
// All of these are HBM- or latency-bound integer/byte work: 128-bit loads and stores where the layout allows,
// warp shuffles for reductions, no tensor cores.
#include "common.cuh"
#include "kernels.cuh"
#include "slots.cuh"

namespace reaxmoe {

// ------------------------------------------------------------------------------------------------------
// K1 route: Gemma-4 routing (vllm/model_executor/models/gemma4.py:183-203; Triton form :95-175).
// One warp per token; lane l holds logits [l*V, l*V + V). Top-k by a total order on (logit, -index): the
// larger logit wins, equal logits go to the lower expert id. -0.0 and +0.0 compare equal.
// w_j = e_j / (e_0 + ... + e_{k-1}) * scale[id_j] with e_j = exp(l_j - l_max): softmax over all experts,
// masked to the top-k and renormalised (the all-expert denominator cancels).
// ------------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t sortable_key(float v) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;  // -0.0 ties with +0.0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int V>
__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ logits, const float* __restrict__ scale,
                                                    int T, int E, int K, int* __restrict__ ids,
                                                    float* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const float* row = logits + t * E;
  float v[V];
  uint64_t key[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int idx = lane * V + i;
    v[i] = idx < E ? row[idx] : 0.0f;
    key[i] = idx < E ? ((uint64_t)sortable_key(v[i]) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)idx) : 0ull;
  }
  int my_id = 0;
  float my_val = 0.0f, top_val = 0.0f;
  for (int j = 0; j < K; ++j) {
    uint64_t best = 0ull;
#pragma unroll
    for (int i = 0; i < V; ++i) best = key[i] > best ? key[i] : best;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const uint64_t o = __shfl_xor_sync(0xffffffffu, best, off);
      best = o > best ? o : best;
    }
    const int id = (int)(0xFFFFFFFFu - (uint32_t)best);
    const int owner = id / V;
    float val = 0.0f;
    if (lane == owner) {
#pragma unroll
      for (int i = 0; i < V; ++i)
        if (lane * V + i == id) { val = v[i]; key[i] = 0ull; }
    }
    val = __shfl_sync(0xffffffffu, val, owner);
    if (j == 0) top_val = val;
    if (lane == j) { my_id = id; my_val = val; }
  }
  const float ex = (lane < K) ? expf(my_val - top_val) : 0.0f;
  float denom = 0.0f;
  for (int j = 0; j < K; ++j) denom = __fadd_rn(denom, __shfl_sync(0xffffffffu, ex, j));
  if (lane < K) {
    float w = __fdiv_rn(ex, denom);
    if (scale != nullptr) w = __fmul_rn(w, scale[my_id]);
    ids[t * K + lane] = my_id;
    weights[t * K + lane] = w;
  }
}

// The same routing with four lanes per token, for batches large enough to fill the GPU that way. A CTA of 128 threads
// (32 tokens) stages its tokens' logits in shared memory, rows padded to a stride of 4 mod 32 words so that the
// quad's reads are free of bank conflicts. Lane q of a token's quad scans the logits q, q + 4, ... keeping its top KMAX
// keys (the 64-bit (logit, -index) order of route_kernel) sorted by a branch-free insertion; the quad then merges its
// four lists in K rounds of a 2-step shuffle maximum. Lane 0 computes the weights with route_kernel's arithmetic and
// summation order: the same ids and weights bit for bit.
constexpr int kRouteTokens = 32;

template <int KMAX>
__global__ void __launch_bounds__(128) route_quad_kernel(const float* __restrict__ logits,
                                                         const float* __restrict__ scale, int T, int E, int K,
                                                         int* __restrict__ ids, float* __restrict__ weights) {
  extern __shared__ float tile[];   // [kRouteTokens][stride]
  const int stride = E + ((4 - E) % 32 + 32) % 32;
  const int64_t t0 = (int64_t)blockIdx.x * kRouteTokens;
  const int nt = (int)((T - t0) < kRouteTokens ? (T - t0) : kRouteTokens);
  {
    // the CTA's rows are nt * E contiguous floats: every thread issues all its loads before its first store, so
    // the loads' DRAM latency is paid once per CTA, not once per row
    constexpr int U = 8;
    const float* src = logits + t0 * E;
    const int total = nt * E;
    if ((E & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      const int n4 = total >> 2;   // stride and E are multiples of 4: a float4 never straddles two rows
      for (int base = threadIdx.x; base < n4; base += blockDim.x * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * blockDim.x;
          if (i < n4) v[u] = __ldg(reinterpret_cast<const float4*>(src) + i);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * blockDim.x;
          if (i < n4) {
            const int tl = (4 * i) / E, e = 4 * i - tl * E;
            *reinterpret_cast<float4*>(tile + tl * stride + e) = v[u];
          }
        }
      }
    } else {
      for (int base = threadIdx.x; base < total; base += blockDim.x * U) {
        float v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * blockDim.x;
          if (i < total) v[u] = __ldg(src + i);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * blockDim.x;
          if (i < total) {
            const int tl = i / E;
            tile[tl * stride + (i - tl * E)] = v[u];
          }
        }
      }
    }
  }
  __syncthreads();
  const int tl = threadIdx.x >> 2, q = threadIdx.x & 3;
  const bool active = tl < nt;
  const float* row = tile + tl * stride;
  uint64_t top[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) top[j] = 0ull;
  if (active) {
    for (int e = q; e < E; e += 4) {
      const uint64_t key = ((uint64_t)sortable_key(row[e]) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)e);
      if (key <= top[KMAX - 1]) continue;
      // insert into the descending list: new[i] = max(old[i], min(old[i-1], key)), new[0] = max(old[0], key)
#pragma unroll
      for (int j = KMAX - 1; j > 0; --j) {
        const uint64_t m = top[j - 1] < key ? top[j - 1] : key;
        top[j] = top[j] > m ? top[j] : m;
      }
      top[0] = top[0] > key ? top[0] : key;
    }
  }
  // merge the quad's lists: K rounds, each takes the largest head and the lane that owned it drops it
  uint64_t win[KMAX];
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < K) {
      uint64_t best = top[0];
      uint64_t o = __shfl_xor_sync(0xffffffffu, best, 1);
      best = o > best ? o : best;
      o = __shfl_xor_sync(0xffffffffu, best, 2);
      best = o > best ? o : best;
      win[j] = best;
      if (top[0] == best) {
#pragma unroll
        for (int i = 0; i < KMAX - 1; ++i) top[i] = top[i + 1];
        top[KMAX - 1] = 0ull;
      }
    }
  }
  if (!active || q != 0) return;
  // weights exactly as route_kernel: e_j = exp(l_j - l_0), denominator summed in increasing j, IEEE division
  const int64_t t = t0 + tl;
  const float top_val = row[(int)(0xFFFFFFFFu - (uint32_t)win[0])];
  float ex[KMAX];
  float denom = 0.0f;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < K) {
      ex[j] = expf(row[(int)(0xFFFFFFFFu - (uint32_t)win[j])] - top_val);
      denom = __fadd_rn(denom, ex[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (j < K) {
      const int id = (int)(0xFFFFFFFFu - (uint32_t)win[j]);
      float w = __fdiv_rn(ex[j], denom);
      if (scale != nullptr) w = __fmul_rn(w, scale[id]);
      ids[t * K + j] = id;
      weights[t * K + j] = w;
    }
  }
}

int launch_route(const float* logits, const float* scale, int T, int E, int K, int* ids, float* w,
                 cudaStream_t s) {
  if (T == 0) return 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = ceil_div64(T, kRouteTokens);
  const size_t smem = (size_t)kRouteTokens * (E + 32) * sizeof(float);
  // four lanes per token once there are enough tokens for several CTAs per SM
  if (blocks >= 4 * sms && K <= 16) {
    if (K <= 8)
      route_quad_kernel<8><<<(unsigned)blocks, 128, smem, s>>>(logits, scale, T, E, K, ids, w);
    else
      route_quad_kernel<16><<<(unsigned)blocks, 128, smem, s>>>(logits, scale, T, E, K, ids, w);
    return 0;
  }
  const int warps_per_block = 8;
  const dim3 grid((unsigned)ceil_div64(T, warps_per_block));
  if (E <= 32) route_kernel<1><<<grid, 256, 0, s>>>(logits, scale, T, E, K, ids, w);
  else if (E <= 64) route_kernel<2><<<grid, 256, 0, s>>>(logits, scale, T, E, K, ids, w);
  else if (E <= 128) route_kernel<4><<<grid, 256, 0, s>>>(logits, scale, T, E, K, ids, w);
  else route_kernel<8><<<grid, 256, 0, s>>>(logits, scale, T, E, K, ids, w);
  return 0;
}

// ------------------------------------------------------------------------------------------------------
// K2a count: per-segment expert histogram (segment = kSegTokens consecutive tokens). Shared-memory integer
// atomics: exact counts, independent of order. A negative id marks an unused slot (the expert-parallel path pads
// a token's experts on another rank with -1) and is skipped; ids >= E are flagged and skipped.
// ------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) count_kernel(const int* __restrict__ ids, int m, int k, int E,
                                                    int* __restrict__ seg_counts, int* status) {
  __shared__ int hist[kMaxExperts];
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int64_t t0 = (int64_t)blockIdx.x * kSegTokens;
  const int n = (int)(kSegTokens < m - t0 ? (int64_t)kSegTokens : m - t0) * k;
  const int* p = ids + t0 * k;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = p[i];
    if ((unsigned)e < (unsigned)E) atomicAdd(&hist[e], 1);
    else if (e >= E) set_status(status, REAXMOE_ERR_BAD_EXPERT_ID);  // negative ids mark unused slots
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) seg_counts[(int64_t)blockIdx.x * E + i] = hist[i];
}

// ------------------------------------------------------------------------------------------------------
// K2b plan: one CTA. Column scan of seg_counts [nseg, E] into seg_base (slots of expert e that precede
// segment s), per-expert counts, expert_offsets[E+1], blockscale_offsets[E+1] (counts rounded up to 128),
// tile_prefix[E+1] (128-row GEMM m-tiles) and, optionally, vLLM's problem_sizes1/2 [E, 3]
// (get_cutlass_moe_mm_data; blink_moe.py:271-299).
// ------------------------------------------------------------------------------------------------------
constexpr int kPlanThreads = 1024;
constexpr int kPlanMaxParts = 32;

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int* __restrict__ seg_counts, int nseg, int E,
                                                            int* __restrict__ seg_base, int* __restrict__ counts,
                                                            int* __restrict__ eoff, int* __restrict__ boff,
                                                            int* __restrict__ tile_prefix, int* ps1, int* ps2,
                                                            int n1, int k1, int n2, int k2) {
  __shared__ int partial[kPlanMaxParts][kMaxExperts];
  __shared__ int total[kMaxExperts];
  const int P = min(kPlanMaxParts, kPlanThreads / E);
  const int e = threadIdx.x % E;
  const int part = threadIdx.x / E;
  const int chunk = (nseg + P - 1) / P;
  const int s0 = part * chunk;
  const int s1 = min(nseg, s0 + chunk);
  if (part < P) {
    int sum = 0;
    for (int s = s0; s < s1; ++s) sum += seg_counts[(int64_t)s * E + e];
    partial[part][e] = sum;
  }
  __syncthreads();
  if (part == 0) {
    int run = 0;
    for (int q = 0; q < P; ++q) {
      const int c = partial[q][e];
      partial[q][e] = run;
      run += c;
    }
    total[e] = run;
  }
  __syncthreads();
  if (part < P) {
    int base = partial[part][e];
    for (int s = s0; s < s1; ++s) {
      const int64_t i = (int64_t)s * E + e;
      const int c = seg_counts[i];
      seg_base[i] = base;
      base += c;
    }
  }
  if (threadIdx.x == 0) {
    int eo = 0, bo = 0, tp = 0;
    for (int x = 0; x < E; ++x) {
      const int c = total[x];
      counts[x] = c;
      eoff[x] = eo;
      boff[x] = bo;
      tile_prefix[x] = tp;
      eo += c;
      bo += (c + 127) / 128 * 128;
      tp += (c + 127) / 128;
    }
    eoff[E] = eo;
    boff[E] = bo;
    tile_prefix[E] = tp;
  }
  if (ps1 != nullptr && threadIdx.x < E) {
    ps1[threadIdx.x * 3 + 0] = total[threadIdx.x];
    ps1[threadIdx.x * 3 + 1] = n1;
    ps1[threadIdx.x * 3 + 2] = k1;
  }
  if (ps2 != nullptr && threadIdx.x < E) {
    ps2[threadIdx.x * 3 + 0] = total[threadIdx.x];
    ps2[threadIdx.x * 3 + 1] = n2;
    ps2[threadIdx.x * 3 + 2] = k2;
  }
}

// ------------------------------------------------------------------------------------------------------
// K3 permute_quant, in two kernels.
//  assign_slots (one warp per segment): canonical slot of every (token, j) pair of the segment, token-major inside
//  an expert, starting from run[e] = expert_offsets[e] + seg_base[seg][e] (segment_slots); writes c_map.
//  quant_scatter (a flat grid of 3 CTAs per SM, one warp per token, tokens strided over all warps): each token row
//  is NVFP4-quantised once per distinct expert input scale and written to its k slots (FP4 bytes + the two scale
//  bytes of each 32-element unit), the same bytes as vLLM's per-slot quant of the shuffled rows
//  (blink_moe.py:301-323, cutlass_moe.py:585-593). The grid does not depend on the segments, so every SM gets the
//  same share of tokens in one wave.
// ------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(32) assign_slots_kernel(const int* __restrict__ ids, const int* __restrict__ seg_base,
                                                         const int* __restrict__ eoff, int m, int E, int k,
                                                         int* __restrict__ c_map) {
  __shared__ int run[kMaxExperts];
  __shared__ uint32_t mask[kMaxExperts];
  __shared__ int pos_s[kSegTokens * kMaxTopk];
  __shared__ short exp_s[kSegTokens * kMaxTopk];
  const int seg = blockIdx.x;
  const int64_t t0 = (int64_t)seg * kSegTokens;
  const int nt = (int)(kSegTokens < m - t0 ? (int64_t)kSegTokens : m - t0);
  for (int e = threadIdx.x; e < E; e += 32) {
    run[e] = eoff[e] + seg_base[(int64_t)seg * E + e];
    mask[e] = 0u;
  }
  __syncwarp();
  segment_slots(ids, t0, nt, k, E, run, mask, pos_s, exp_s, c_map);
}

constexpr int kQuantCtasPerSm = 3;

// Lanes j < k put slot j and its input scale into the warp's shared slot table; lanes own 32-element units (16 FP4
// bytes + 2 scale bytes per slot). A unit is quantised once per distinct input scale among the slots (once for a
// uniform scale) with the bf16x2 quantiser, then stored to every slot: FP4 bytes into the slot's row, scale bytes
// into the slot's row of the linear scale buffer (full-sector stores; the atoms are written from it by
// swizzle_scales_kernel).
// Gather layout (tok_fp4 != nullptr): when every expert has the same input scale, the quantised row is the same for
// all of a token's slots, so it is stored once, token-major: FP4 bytes into tok_fp4 [m, H/2] and scale bytes into
// tok_sf [m, H/16]; row_token[slot] = token lets the w13 GEMM and the scale swizzle fetch a slot's row by its token.
// *ga_flag (written by CTA 0) records which layout was written: 1 token-major, 0 per slot (scales differ).
__global__ void __launch_bounds__(256, kQuantCtasPerSm) quant_scatter_kernel(
    const __nv_bfloat16* __restrict__ a, const float* __restrict__ a1_gscale, const int* __restrict__ ids,
    const int* __restrict__ c_map, int m, int H, int E, int k, uint8_t* __restrict__ rep_fp4,
    uint8_t* __restrict__ lin_sf, uint8_t* __restrict__ tok_fp4, uint8_t* __restrict__ tok_sf,
    int* __restrict__ row_token, int* __restrict__ ga_flag) {
  __shared__ float gq[kMaxExperts];
  __shared__ int sl_pos[8][kMaxTopk];           // per warp: the current token's slots
  __shared__ float sl_g[8][kMaxTopk];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) gq[e] = __fdiv_rn(1.0f, a1_gscale[e]);
  __syncthreads();
  bool same = true;
  for (int e = threadIdx.x; e < E; e += blockDim.x) same = same && __float_as_uint(gq[e]) == __float_as_uint(gq[0]);
  const bool ga = __syncthreads_and(same ? 1 : 0) != 0 && tok_fp4 != nullptr;
  if (tok_fp4 != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *ga_flag = ga ? 1 : 0;
  const int units = H / 32;
  const int k16 = H / 16;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int t = blockIdx.x * (blockDim.x >> 5) + warp; t < m; t += nwarps) {
    const uint4* src = reinterpret_cast<const uint4*>(a + (int64_t)t * H);
    uint4 raw[kPermUnits][4];
#pragma unroll
    for (int it = 0; it < kPermUnits; ++it) {
      const int un = lane + 32 * it;
      if (un < units) {
#pragma unroll
        for (int i = 0; i < 4; ++i) raw[it][i] = __ldg(src + un * 4 + i);
      }
    }
    if (ga) {
      if (lane < k) {
        const int pos = c_map[(int64_t)t * k + lane];
        if (pos >= 0) row_token[pos] = (int)t;
      }
      const float g = gq[0];
#pragma unroll
      for (int it = 0; it < kPermUnits; ++it) {
        const int un = lane + 32 * it;
        if (un >= units) continue;
        uint32_t w[4];
        uint32_t sb = 0u;
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const uint4 q0 = raw[it][2 * b], q1 = raw[it][2 * b + 1];
          const uint32_t xw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
          sb |= quant_block16_bf16(xw, g, w[2 * b], w[2 * b + 1]) << (8 * b);
        }
        *reinterpret_cast<uint4*>(tok_fp4 + (int64_t)t * (H / 2) + un * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint16_t*>(tok_sf + (int64_t)t * k16 + un * 2) = (uint16_t)sb;
      }
      continue;
    }
    if (lane < k) {
      const int64_t pair = (int64_t)t * k + lane;
      const int pos = c_map[pair];   // -1 for an id outside [0, E)
      sl_pos[warp][lane] = pos;
      sl_g[warp][lane] = pos >= 0 ? gq[ids[pair]] : 0.0f;
    }
    __syncwarp();
#pragma unroll
    for (int it = 0; it < kPermUnits; ++it) {
      const int un = lane + 32 * it;
      if (un >= units) continue;
      uint32_t w[4];
      uint32_t sb = 0u;
      uint32_t gbits = 0xFFFFFFFFu;  // a NaN pattern: never equal to a real scale
      for (int j = 0; j < k; ++j) {
        const int pos = sl_pos[warp][j];
        if (pos < 0) continue;
        const float g = sl_g[warp][j];
        if (__float_as_uint(g) != gbits) {
          gbits = __float_as_uint(g);
          sb = 0u;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint4 q0 = raw[it][2 * b], q1 = raw[it][2 * b + 1];
            const uint32_t xw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            sb |= quant_block16_bf16(xw, g, w[2 * b], w[2 * b + 1]) << (8 * b);
          }
        }
        *reinterpret_cast<uint4*>(rep_fp4 + (int64_t)pos * (H / 2) + un * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint16_t*>(lin_sf + (int64_t)pos * k16 + un * 2) = (uint16_t)sb;
      }
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------------------------------------
// K3a' permute_fp4: the same slot assignment as permute_quant, for token rows that are already NVFP4 (a fused
// norm + quantise upstream, e.g. add + RMSNorm + quant in one kernel as engine/fp4_triton.py:68-90 does): each slot
// receives a byte copy of its token's FP4 row and linear scale row. The copy is exact only if every slot's expert
// quantises with the scale the rows were made with (a1_gscale[e] == in_gscale); a slot whose expert differs flags
// REAXMOE_ERR_UNSUPPORTED in the status word and is copied all the same. Gather layout (row_token != nullptr): no
// copies; row_token[slot] = token, and the w13 GEMM and the scale swizzle read the token rows in place.
// ------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) permute_fp4_kernel(
    const uint8_t* __restrict__ a_fp4, const uint8_t* __restrict__ a_sf, float in_gscale,
    const float* __restrict__ a1_gscale, const int* __restrict__ ids, const int* __restrict__ seg_base,
    const int* __restrict__ eoff, int m, int H, int E, int k, uint8_t* __restrict__ rep_fp4,
    uint8_t* __restrict__ lin_sf, int* __restrict__ c_map, int* status, int* __restrict__ row_token,
    int* __restrict__ ga_flag) {
  __shared__ int run[kMaxExperts];
  __shared__ uint32_t mask[kMaxExperts];
  __shared__ int pos_s[kSegTokens * kMaxTopk];
  __shared__ short exp_s[kSegTokens * kMaxTopk];
  const int seg = blockIdx.x;
  const int64_t t0 = (int64_t)seg * kSegTokens;
  const int nt = (int)(kSegTokens < m - t0 ? (int64_t)kSegTokens : m - t0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    run[e] = eoff[e] + seg_base[(int64_t)seg * E + e];
    mask[e] = 0u;
  }
  __syncthreads();
  if (warp == 0) segment_slots(ids, t0, nt, k, E, run, mask, pos_s, exp_s, c_map);
  __syncthreads();
  if (row_token != nullptr) {
    // gather layout: the token rows stay where they are; each slot records its token
    if (seg == 0 && threadIdx.x == 0) *ga_flag = 1;
    for (int i = threadIdx.x; i < nt * k; i += blockDim.x) {
      const int e = exp_s[i];
      if (e < 0) continue;
      row_token[pos_s[i]] = (int)(t0 + i / k);
      if (a1_gscale[e] != in_gscale) set_status(status, REAXMOE_ERR_UNSUPPORTED);
    }
    return;
  }
  const int row16 = H / 32;          // 16-byte pieces of an FP4 row
  const int sf16 = H / 256;          // 16-byte pieces of a linear scale row
  constexpr int kMaxRow = 4;         // H <= 4096: <= 128 pieces, 4 per lane
  for (int tl = warp; tl < nt; tl += blockDim.x >> 5) {
    const int64_t t = t0 + tl;
    const uint4* src = reinterpret_cast<const uint4*>(a_fp4 + t * (H / 2));
    uint4 row[kMaxRow];
#pragma unroll
    for (int i = 0; i < kMaxRow; ++i)
      if (lane + 32 * i < row16) row[i] = __ldg(src + lane + 32 * i);
    uint4 sfv = make_uint4(0u, 0u, 0u, 0u);
    if (lane < sf16) sfv = __ldg(reinterpret_cast<const uint4*>(a_sf + t * (H / 16)) + lane);
    for (int j = 0; j < k; ++j) {
      const int e = exp_s[tl * k + j];
      if (e < 0) continue;
      const int64_t pos = pos_s[tl * k + j];
      if (lane == 0 && a1_gscale[e] != in_gscale) set_status(status, REAXMOE_ERR_UNSUPPORTED);
      uint4* dst = reinterpret_cast<uint4*>(rep_fp4 + pos * (H / 2));
#pragma unroll
      for (int i = 0; i < kMaxRow; ++i)
        if (lane + 32 * i < row16) dst[lane + 32 * i] = row[i];
      if (lane < sf16) reinterpret_cast<uint4*>(lin_sf + pos * (H / 16))[lane] = sfv;
    }
  }
}

// ------------------------------------------------------------------------------------------------------
// K3b swizzle_scales: one CTA per GEMM m-tile gm (expert e, 128 routed rows), whose scale rows are atom row block gm
// of the 128x4 layout (blockscale_offsets[e] / 128 == tile_prefix[e]). Reads the tile's rows of the linear scale
// buffer [slots, H/16] (contiguous) into shared memory and writes its H/64 atoms of 512 bytes with 16-byte stores
// (atom row i = the 4 scale bytes of rows i, i+32, i+64, i+96). Rows past the expert's count are written as zero.
// Gather layout (row_map != nullptr and *ga_flag set): the scale rows are read from the token-major rows of tok
// (tok_stride bytes apart: H/16 for packed scale rows, the record size for expert-parallel records), row r of the
// tile from row row_map[slot]; otherwise from lin.
// ------------------------------------------------------------------------------------------------------
constexpr int kSwzMaxWords = 128 * (48 + 1);   // 128 rows x (H/64 <= 48 words + 1 pad word)

__global__ void __launch_bounds__(256) swizzle_scales_kernel(const uint8_t* __restrict__ lin,
                                                             const int* __restrict__ tile_prefix,
                                                             const int* __restrict__ counts,
                                                             const int* __restrict__ eoff, int E, int H,
                                                             uint8_t* __restrict__ sf,
                                                             const int* __restrict__ row_map,
                                                             const int* __restrict__ ga_flag,
                                                             const uint8_t* __restrict__ tok, int tok_rows,
                                                             int64_t tok_stride) {
  __shared__ uint32_t tile[kSwzMaxWords];
  const int gm = blockIdx.x;
  if (gm >= tile_prefix[E]) return;
  int lo = 0, hi = E;  // largest e with tile_prefix[e] <= gm
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tile_prefix[mid] <= gm) lo = mid; else hi = mid;
  }
  const int e = lo;
  const int mt = gm - tile_prefix[e];
  const int rows = min(128, counts[e] - mt * 128);
  const int k64 = H / 64;             // 4-byte words per row
  const int stride = k64 + 1;         // odd: conflict-free column reads
  // vector loads: 16 bytes when a row of H/16 scale bytes is a multiple of 16 (H % 256 == 0), else 8 bytes (H is a
  // multiple of 128); stored as words at the odd stride
  const uint8_t* src = lin + ((int64_t)eoff[e] + mt * 128) * (H / 16);
  if (row_map != nullptr && *ga_flag != 0) {
    // gather layout: row r of the tile is token row_map[slot] of the token-major scale rows
    const int* rm = row_map + eoff[e] + mt * 128;
    const int k128 = k64 / 2;
    for (int i = threadIdx.x; i < 128 * k128; i += blockDim.x) {
      const int r = i / k128, c = (i - r * k128) * 2;
      uint2 v = make_uint2(0u, 0u);
      if (r < rows) {
        const int t = min(max(__ldg(rm + r), 0), tok_rows - 1);   // clamped: never outside the token rows
        v = __ldg(reinterpret_cast<const uint2*>(tok + (int64_t)t * tok_stride) + (i - r * k128));
      }
      uint32_t* d = tile + r * stride + c;
      d[0] = v.x;
      d[1] = v.y;
    }
  } else if (k64 % 4 == 0) {
    const int k256 = k64 / 4;
    for (int i = threadIdx.x; i < 128 * k256; i += blockDim.x) {
      const int r = i / k256, c = (i - r * k256) * 4;
      const uint4 v = r < rows ? __ldg(reinterpret_cast<const uint4*>(src) + i) : make_uint4(0u, 0u, 0u, 0u);
      uint32_t* d = tile + r * stride + c;
      d[0] = v.x;
      d[1] = v.y;
      d[2] = v.z;
      d[3] = v.w;
    }
  } else {
    const int k128 = k64 / 2;
    for (int i = threadIdx.x; i < 128 * k128; i += blockDim.x) {
      const int r = i / k128, c = (i - r * k128) * 2;
      const uint2 v = r < rows ? __ldg(reinterpret_cast<const uint2*>(src) + i) : make_uint2(0u, 0u);
      uint32_t* d = tile + r * stride + c;
      d[0] = v.x;
      d[1] = v.y;
    }
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(sf + (int64_t)gm * k64 * 512);
  for (int i = threadIdx.x; i < k64 * 32; i += blockDim.x) {
    const int kc = i >> 5, q = i & 31;
    dst[i] = make_uint4(tile[q * stride + kc], tile[(q + 32) * stride + kc], tile[(q + 64) * stride + kc],
                        tile[(q + 96) * stride + kc]);
  }
}

int launch_swizzle_scales(const uint8_t* lin, const int* tile_prefix, const int* counts, const int* eoff, int E, int H,
                          int64_t slots, uint8_t* sf, cudaStream_t s, const int* row_map, const int* ga_flag,
                          const uint8_t* tok_sf, int tok_rows, int64_t tok_stride) {
  if (slots == 0) return 0;
  const int64_t max_tiles = slots / 128 + E + 1;
  swizzle_scales_kernel<<<(unsigned)max_tiles, 256, 0, s>>>(lin, tile_prefix, counts, eoff, E, H, sf, row_map,
                                                            ga_flag, tok_sf, tok_rows,
                                                            tok_stride > 0 ? tok_stride : (int64_t)(H / 16));
  return 0;
}

// ------------------------------------------------------------------------------------------------------
// K7 combine: one warp per token, 8 columns (one 16-byte load per slot row) per lane step.
// out = bf16( sum_j bf16( c3[c_map[t,j]] * bf16(w[t,j]) ) ), partial sums j % 4 in increasing j, then
// ((s0 + s1) + s2) + s3 (blink_moe.py:168-198 ORDER 1 for top-8; cutlass_moe.py:650-662).
// The compile-time-k variant issues all k row loads of two lane steps before any arithmetic, so 2k 16-byte
// loads per lane are in flight; other k use the runtime-k loop.
// ------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void combine_accumulate(const uint4& v, float wb, int j, float (&part)[4][8]) {
  float f[8];
  bf16x8_to_f32(v, f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float p = bf16r(__fmul_rn(f[i], wb));
    part[j & 3][i] = (j < 4) ? p : __fadd_rn(part[j & 3][i], p);
  }
}
__device__ __forceinline__ uint4 combine_finish(float (&part)[4][8], int k) {
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i] = part[0][i];
    if (k > 1) acc[i] = __fadd_rn(acc[i], part[1][i]);
    if (k > 2) acc[i] = __fadd_rn(acc[i], part[2][i]);
    if (k > 3) acc[i] = __fadd_rn(acc[i], part[3][i]);
  }
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  return o;
}

// Where row t goes: PlainRows writes out[t]; RoutedRows sends the row of record t to its source rank's return buffer
// (RowRoute; a peer's memory over NVLink or this GPU's own) and fences the stores at system scope before the thread
// exits, so that a following ep_signal_kernel publishes them.
struct PlainRows {
  static constexpr bool kPeer = false;
  __nv_bfloat16* out;
  __device__ __forceinline__ uint4* row(int64_t t, int H) const { return reinterpret_cast<uint4*>(out + t * H); }
  __device__ __forceinline__ bool skip(int) const { return false; }
};
struct RoutedRows {
  static constexpr bool kPeer = true;
  RowRoute r;
  __device__ __forceinline__ uint4* row(int64_t t, int H) const { return reinterpret_cast<uint4*>(r.row_addr(t, H)); }
  __device__ __forceinline__ bool skip(int valid_pairs) const { return r.skip_single && valid_pairs == 1; }
};

template <int K, class Rows, int THREADS = 256, int MIN_BLOCKS = 3>
__global__ void __launch_bounds__(THREADS, MIN_BLOCKS) combine_kernel_k(const __nv_bfloat16* __restrict__ c3,
                                                                        const int* __restrict__ c_map,
                                                                        const float* __restrict__ topk_w, int m,
                                                                        int H, const __grid_constant__ Rows out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nch = H / 8;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < m; t += warps) {
    int mypos = 0;
    float myw = 0.0f;
    if (lane < K) {
      mypos = c_map[t * K + lane];
      // an unmapped pair (no slot) adds exactly +0: its weight is taken as +0, whatever the router gave it
      myw = mypos >= 0 ? bf16r(topk_w[t * K + lane]) : 0.0f;
    }
    const uint4* rowp[K];
    float wb[K];
    bool valid[K];
    int nvalid = 0;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int pj = __shfl_sync(0xffffffffu, mypos, j);
      wb[j] = __shfl_sync(0xffffffffu, myw, j);
      valid[j] = pj >= 0;  // -1 marks a pair whose expert id was out of range (flagged by the plan)
      nvalid += valid[j] ? 1 : 0;
      rowp[j] = reinterpret_cast<const uint4*>(c3 + (int64_t)(valid[j] ? pj : 0) * H);
    }
    if (out.skip(nvalid)) continue;
    uint4* orow = out.row(t, H);
    for (int ch = lane; ch < nch; ch += 32) {
      uint4 v[K];
#pragma unroll
      for (int j = 0; j < K; ++j) v[j] = valid[j] ? __ldg(rowp[j] + ch) : make_uint4(0u, 0u, 0u, 0u);
      float part[4][8];
#pragma unroll
      for (int j = 0; j < K; ++j) combine_accumulate(v[j], wb[j], j, part);
      orow[ch] = combine_finish(part, K);
    }
  }
  if (Rows::kPeer) __threadfence_system();
}

template <class Rows>
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ c3,
                                                      const int* __restrict__ c_map,
                                                      const float* __restrict__ topk_w, int m, int H, int k,
                                                      const __grid_constant__ Rows out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < m; t += warps) {
    int mypos = 0;
    float myw = 0.0f;
    if (lane < k) {
      mypos = c_map[t * k + lane];
      myw = mypos >= 0 ? bf16r(topk_w[t * k + lane]) : 0.0f;   // an unmapped pair adds exactly +0
    }
    int pos[kMaxTopk];
    float wb[kMaxTopk];
    int nvalid = 0;
#pragma unroll
    for (int j = 0; j < kMaxTopk; ++j) {
      pos[j] = __shfl_sync(0xffffffffu, mypos, j);
      wb[j] = __shfl_sync(0xffffffffu, myw, j);
      nvalid += (j < k && pos[j] >= 0) ? 1 : 0;
    }
    if (out.skip(nvalid)) continue;
    for (int ch = lane; ch < H / 8; ch += 32) {
      float part[4][8];
#pragma unroll
      for (int j = 0; j < kMaxTopk; ++j) {
        if (j < k) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (pos[j] >= 0) v = __ldg(reinterpret_cast<const uint4*>(c3 + (int64_t)pos[j] * H) + ch);
          combine_accumulate(v, wb[j], j, part);
        }
      }
      out.row(t, H)[ch] = combine_finish(part, k);
    }
  }
  if (Rows::kPeer) __threadfence_system();
}

// ------------------------------------------------------------------------------------------------------
// NVFP4 quantisation of rows (engine/fp4.py::quantize_nvfp4 numerics; fp4_triton.py nvfp4_quant_static).
// One warp per row, one 64-element group (4 scale blocks) per lane step.
// ------------------------------------------------------------------------------------------------------
template <bool F32>
__global__ void __launch_bounds__(256) quantize_kernel(const void* __restrict__ x, int64_t rows, int cols,
                                                       int group_rows, const float* __restrict__ gscale,
                                                       uint8_t* __restrict__ packed, uint8_t* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t grp_id = r / group_rows;
  const int64_t sfrow = grp_id * ((group_rows + 127) / 128 * 128) + (r - grp_id * group_rows);
  const float g = __fdiv_rn(1.0f, gscale[grp_id]);
  const int k64 = cols / 64;
  for (int grp = lane; grp < cols / 64; grp += 32) {
    float v[64];
    if constexpr (F32) {
      const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(x) + r * cols) + grp * 16;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 q = __ldg(src + i);
        v[4 * i] = q.x; v[4 * i + 1] = q.y; v[4 * i + 2] = q.z; v[4 * i + 3] = q.w;
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(x) + r * cols) + grp * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) bf16x8_to_f32(__ldg(src + i), v + 8 * i);
    }
    uint32_t w[8];
    uint32_t sbytes = 0u;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      float blk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) blk[i] = v[b * 16 + i];
      sbytes |= quant_block16(blk, g, w[2 * b], w[2 * b + 1]) << (8 * b);
    }
    uint4* dst = reinterpret_cast<uint4*>(packed + r * (cols / 2) + grp * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    *reinterpret_cast<uint32_t*>(scales + sf_offset(sfrow, grp * 4, k64)) = sbytes;
  }
}

int launch_quantize(const void* x, bool f32, int64_t rows, int cols, int group_rows, const float* gscale,
                    uint8_t* packed, uint8_t* scales, cudaStream_t s) {
  if (rows == 0) return 0;
  const dim3 grid((unsigned)ceil_div64(rows, 8));
  if (f32) quantize_kernel<true><<<grid, 256, 0, s>>>(x, rows, cols, group_rows, gscale, packed, scales);
  else quantize_kernel<false><<<grid, 256, 0, s>>>(x, rows, cols, group_rows, gscale, packed, scales);
  return 0;
}

// ------------------------------------------------------------------------------------------------------
// w13 prepack: output row block b (256 rows; the last one narrower when inter % 128 != 0) holds the gate rows of
// intermediate columns [128b, 128b + h) then the matching up rows inter + [128b, 128b + h), h = min(128,
// inter - 128b): output row r = 256b + w <- gate row 128b + w (w < h) or up row inter + 128b + (w - h). Its
// 16-element block scales move with it.
// ------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(128) prepack_w13_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sf,
                                                          int inter, int H, uint8_t* __restrict__ wp,
                                                          uint8_t* __restrict__ sfp) {
  const int N = 2 * inter;
  const int e = blockIdx.y;
  const int r = blockIdx.x;
  const int b = r >> 8, wi = r & 255;
  const int h = min(128, inter - 128 * b);
  const int src = wi < h ? 128 * b + wi : inter + 128 * b + (wi - h);
  const int64_t row_bytes = H / 2;
  const uint4* s4 = reinterpret_cast<const uint4*>(w + ((int64_t)e * N + src) * row_bytes);
  uint4* d4 = reinterpret_cast<uint4*>(wp + ((int64_t)e * N + r) * row_bytes);
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d4[i] = s4[i];
  const int k64 = H / 64;
  const int64_t esz = (int64_t)(N / 128) * k64 * 512;
  for (int kb = threadIdx.x; kb < H / 16; kb += blockDim.x)
    sfp[e * esz + sf_offset(r, kb, k64)] = sf[e * esz + sf_offset(src, kb, k64)];
}

int launch_prepack_w13(const uint8_t* w, const uint8_t* sf, int E, int inter, int H, uint8_t* wp, uint8_t* sfp,
                       cudaStream_t s) {
  prepack_w13_kernel<<<dim3(2 * inter, E), 128, 0, s>>>(w, sf, inter, H, wp, sfp);
  return 0;
}

int launch_count(const int* ids, int m, int k, int E, int* seg_counts, int* status, cudaStream_t s) {
  const int nseg = (int)ceil_div64(m, kSegTokens);
  if (nseg > 0) count_kernel<<<nseg, 256, 0, s>>>(ids, m, k, E, seg_counts, status);
  return 0;
}

int launch_plan(const int* seg_counts, int nseg, int E, int* seg_base, int* counts, int* eoff, int* boff,
                int* tile_prefix, int* ps1, int* ps2, int n1, int k1, int n2, int k2, cudaStream_t s) {
  plan_kernel<<<1, kPlanThreads, 0, s>>>(seg_counts, nseg, E, seg_base, counts, eoff, boff, tile_prefix, ps1, ps2,
                                         n1, k1, n2, k2);
  return 0;
}

int launch_permute_quant(const __nv_bfloat16* a, const float* a1_gscale, const int* ids, const int* seg_base,
                         const int* eoff, const int* boff, int m, int H, int E, int k, uint8_t* rep_fp4,
                         uint8_t* lin_sf, int* c_map, cudaStream_t s, const GatherRows* ga) {
  (void)boff;
  if (m == 0) return 0;
  const int nseg = (int)ceil_div64(m, kSegTokens);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  assign_slots_kernel<<<nseg, 32, 0, s>>>(ids, seg_base, eoff, m, E, k, c_map);
  const int64_t want = ceil_div64(m, 8), cap = (int64_t)kQuantCtasPerSm * sms;
  quant_scatter_kernel<<<(unsigned)(want < cap ? want : cap), 256, 0, s>>>(
      a, a1_gscale, ids, c_map, m, H, E, k, rep_fp4, lin_sf, ga ? ga->tok_fp4 : nullptr, ga ? ga->tok_sf : nullptr,
      ga ? ga->row_token : nullptr, ga ? ga->flag : nullptr);
  return 0;
}

int launch_permute_fp4(const uint8_t* a_fp4, const uint8_t* a_sf, float in_gscale, const float* a1_gscale,
                       const int* ids, const int* seg_base, const int* eoff, int m, int H, int E, int k,
                       uint8_t* rep_fp4, uint8_t* lin_sf, int* c_map, int* status, cudaStream_t s,
                       const GatherRows* ga) {
  const int nseg = (int)ceil_div64(m, kSegTokens);
  if (nseg > 0)
    permute_fp4_kernel<<<nseg, 256, 0, s>>>(a_fp4, a_sf, in_gscale, a1_gscale, ids, seg_base, eoff, m, H, E, k,
                                            rep_fp4, lin_sf, c_map, status, ga ? ga->row_token : nullptr,
                                            ga ? ga->flag : nullptr);
  return 0;
}

template <class Rows>
static void launch_combine_rows(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                                const Rows& out, unsigned blocks, cudaStream_t s) {
  if (k == 8) combine_kernel_k<8, Rows><<<blocks, 256, 0, s>>>(c3, c_map, w, m, H, out);
  else if (k == 4) combine_kernel_k<4, Rows><<<blocks, 256, 0, s>>>(c3, c_map, w, m, H, out);
  else if (k == 2) combine_kernel_k<2, Rows><<<blocks, 256, 0, s>>>(c3, c_map, w, m, H, out);
  else if (k == 1) combine_kernel_k<1, Rows><<<blocks, 256, 0, s>>>(c3, c_map, w, m, H, out);
  else combine_kernel<Rows><<<blocks, 256, 0, s>>>(c3, c_map, w, m, H, k, out);
}

int launch_combine(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                   __nv_bfloat16* out, int num_sms, cudaStream_t s) {
  if (m == 0) return 0;
  const int64_t want = ceil_div64(m, 8), cap = (int64_t)num_sms * 12;
  const int64_t blocks = want < cap ? want : cap;
  launch_combine_rows(c3, c_map, w, m, H, k, PlainRows{out}, (unsigned)blocks, s);
  return 0;
}

// The routed pre-sum on exactly `sms` SMs, beside a persistent kernel that holds the others: one 1024-thread block per
// SM, made to own its SM by a 64 KiB shared-memory reservation (with it no grouped-GEMM CTA fits on the same SM, and
// no second block of this kernel). K = 8 / 4 / 2 / 1 only.
int launch_combine_routed_pinned(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                                 const RowRoute& route, int sms, cudaStream_t s) {
  if (m == 0) return 0;
  constexpr int kReserve = 64 * 1024;
  const RoutedRows out{route};
  const int64_t want = ceil_div64(m, 32);
  const unsigned blocks = (unsigned)(want < sms ? want : sms);
#define REAXMOE_PINNED(KK)                                                                                          \
  {                                                                                                                 \
    auto fn = combine_kernel_k<KK, RoutedRows, 1024, 1>;                                                            \
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kReserve) != cudaSuccess) return 1;   \
    fn<<<blocks, 1024, kReserve, s>>>(c3, c_map, w, m, H, out);                                                     \
    return 0;                                                                                                       \
  }
  if (k == 8) REAXMOE_PINNED(8)
  if (k == 4) REAXMOE_PINNED(4)
  if (k == 2) REAXMOE_PINNED(2)
  if (k == 1) REAXMOE_PINNED(1)
#undef REAXMOE_PINNED
  return launch_combine_routed(c3, c_map, w, m, H, k, route, sms, s);
}

int launch_combine_routed(const __nv_bfloat16* c3, const int* c_map, const float* w, int m, int H, int k,
                          const RowRoute& route, int num_sms, cudaStream_t s) {
  if (m == 0) return 0;
  const int64_t want = ceil_div64(m, 8), cap = (int64_t)num_sms * 12;
  const int64_t blocks = want < cap ? want : cap;
  launch_combine_rows(c3, c_map, w, m, H, k, RoutedRows{route}, (unsigned)blocks, s);
  return 0;
}

}  // namespace reaxmoe
