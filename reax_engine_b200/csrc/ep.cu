// ep.cu -- expert-parallel dispatch / receive / combine kernels.
//
// Rank r of R owns experts [r*El, (r+1)*El), El = E / R. A token is sent once to every rank that owns at least one
// of its k experts, as one fixed-size record:
//   [0, H/2)                 NVFP4 codes of the token row (element 2i in the low nibble of byte i)
//   [H/2, H/2 + H/16)        e4m3 scale of 16-element block b at byte H/2 + b (linear, not swizzled)
//   [M, M + 4k)              int32 local expert id of pair j (id - r*El), or -1 when expert j is on another rank
//   [M + 4k, M + 8k)         fp32 router weight of pair j
//   padding to a multiple of 16 bytes;                    M = H/2 + H/16.
// The row is quantised with the input scale of the destination rank (a1_gscale must be constant over each rank's
// experts: the quantise-once-then-dispatch contract of vLLM's naive EP prepare, prepare_finalize/naive_dp_ep.py:
// 16-52, which also ships unswizzled scales and swizzles them after the exchange). The receiver places the records'
// pairs into expert-sorted slots, runs the grouped GEMMs and pre-sums each record's local pairs into one bf16 row
// (the combine of the single-GPU layer restricted to the local pairs); the source adds the returned rows of a token
// in fp32 in increasing j of each rank's first pair and rounds once to bf16.
// All of this is HBM/latency-bound byte work: 128-bit loads and stores, no tensor cores.
#include "common.cuh"
#include "kernels.cuh"
#include "slots.cuh"

namespace reaxmoe {

// Rank id of each (token, j) pair for the dispatch plan: the owner rank of expert ids[t, j] for the first pair of
// the token on that rank, -1 for later pairs on the same rank and for negative (unused) ids, R for ids >= E (the
// count kernel flags those). Block 0 also checks that a1_gscale is constant over each rank's experts.
__global__ void __launch_bounds__(256) ep_rank_ids_kernel(const int* __restrict__ ids, int m, int k, int E, int El,
                                                          const float* __restrict__ a1_gscale, int* __restrict__ rid,
                                                          int* status) {
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (__float_as_uint(a1_gscale[e]) != __float_as_uint(a1_gscale[(e / El) * El]))
        set_status(status, REAXMOE_ERR_UNSUPPORTED);
  }
  const int R = E / El;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= m) return;
  int own[kMaxTopk];
#pragma unroll
  for (int j = 0; j < kMaxTopk; ++j) {
    if (j >= k) break;
    const int e = ids[t * k + j];
    int r = e < 0 ? -1 : (e >= E ? R : e / El);
    own[j] = r;
    if (r >= 0 && r < R) {
#pragma unroll
      for (int q = 0; q < kMaxTopk; ++q)
        if (q < j && own[q] == r) r = -1;
    }
    rid[t * k + j] = r;
  }
}

// Dispatch pack: one CTA per segment of kSegTokens tokens. Phase A (warp 0) gives every first pair of a
// (token, rank) its record index, token-major inside a rank's contiguous range; send_map [m, k] gets the record
// index at that pair and -1 elsewhere. Phase B quantises each token row once per distinct rank scale and writes its
// records.
//
// kPeer: the records go straight to their destinations, dst.p[r] being the address of this rank's first record in
// rank r's receive buffer (a peer's memory over NVLink, or this GPU's own); `records` is unused. Every thread fences
// its stores at system scope before it exits, so a following ep_signal_kernel publishes them.
template <bool kPeer>
__global__ void __launch_bounds__(256, 3) ep_pack_kernel(
    const __nv_bfloat16* __restrict__ a, const float* __restrict__ a1_gscale, const int* __restrict__ ids,
    const float* __restrict__ topk_w, const int* __restrict__ rid, const int* __restrict__ seg_base,
    const int* __restrict__ roff, int m, int H, int E, int El, int k, int rec_bytes, uint8_t* __restrict__ records,
    int* __restrict__ send_map, const PeerPtrs dst) {
  __shared__ int run[kMaxRanks];
  __shared__ int roff_s[kMaxRanks];
  __shared__ uint32_t mask[kMaxRanks];
  __shared__ float gq[kMaxRanks];
  __shared__ int pos_s[kSegTokens * kMaxTopk];
  __shared__ short rank_s[kSegTokens * kMaxTopk];
  const int R = E / El;
  const int seg = blockIdx.x;
  const int64_t t0 = (int64_t)seg * kSegTokens;
  const int nt = (int)(kSegTokens < m - t0 ? (int64_t)kSegTokens : m - t0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    roff_s[r] = roff[r];
    run[r] = roff[r] + seg_base[(int64_t)seg * R + r];
    mask[r] = 0u;
    gq[r] = __fdiv_rn(1.0f, a1_gscale[r * El]);
  }
  __syncthreads();
  if (warp == 0) segment_slots(rid, t0, nt, k, R, run, mask, pos_s, rank_s, send_map);
  __syncthreads();
  const int units = H / 32;
  const int meta = H / 2 + H / 16;
  const int nwarps = blockDim.x >> 5;
  constexpr int kMaxUnits = kPermUnits;
  for (int tl = warp; tl < nt; tl += nwarps) {
    const int64_t t = t0 + tl;
    const uint4* src = reinterpret_cast<const uint4*>(a + t * H);
    uint4 raw[kMaxUnits][4];
#pragma unroll
    for (int it = 0; it < kMaxUnits; ++it) {
      const int un = lane + 32 * it;
      if (un < units) {
#pragma unroll
        for (int i = 0; i < 4; ++i) raw[it][i] = __ldg(src + un * 4 + i);
      }
    }
    // metadata: lane j < k holds pair j
    int my_id = -1;
    float my_w = 0.0f;
    if (lane < k) {
      my_id = ids[t * k + lane];
      my_w = topk_w[t * k + lane];
    }
    for (int j = 0; j < k; ++j) {
      const int r = rank_s[tl * k + j];
      if (r < 0) continue;
      uint8_t* rec = kPeer ? reinterpret_cast<uint8_t*>(dst.p[r]) + (int64_t)(pos_s[tl * k + j] - roff_s[r]) * rec_bytes
                           : records + (int64_t)pos_s[tl * k + j] * rec_bytes;
      if (lane < k) {
        const int lid = ((unsigned)my_id < (unsigned)E && my_id / El == r) ? my_id - r * El : -1;
        reinterpret_cast<int*>(rec + meta)[lane] = lid;
        reinterpret_cast<float*>(rec + meta + 4 * k)[lane] = my_w;
      }
    }
#pragma unroll
    for (int it = 0; it < kMaxUnits; ++it) {
      const int un = lane + 32 * it;
      if (un >= units) continue;
      uint32_t w[4];
      uint32_t sbytes = 0u;
      uint32_t gbits = 0xFFFFFFFFu;  // a NaN pattern: never equal to a real scale
      for (int j = 0; j < k; ++j) {
        const int r = rank_s[tl * k + j];
        if (r < 0) continue;
        const float g = gq[r];
        if (__float_as_uint(g) != gbits) {
          gbits = __float_as_uint(g);
          sbytes = 0u;
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint4 q0 = raw[it][2 * b], q1 = raw[it][2 * b + 1];
            const uint32_t xw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            sbytes |= quant_block16_bf16(xw, g, w[2 * b], w[2 * b + 1]) << (8 * b);
          }
        }
        uint8_t* rec = kPeer ? reinterpret_cast<uint8_t*>(dst.p[r]) +
                                   (int64_t)(pos_s[tl * k + j] - roff_s[r]) * rec_bytes
                             : records + (int64_t)pos_s[tl * k + j] * rec_bytes;
        *reinterpret_cast<uint4*>(rec + un * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint16_t*>(rec + H / 2 + un * 2) = (uint16_t)sbytes;
      }
    }
  }
  if (kPeer) __threadfence_system();
}

__device__ __forceinline__ uint64_t clock_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Cross-rank signal (a barrier with an optional payload), one CTA of kMaxRanks threads. Thread d < ranks: when
// `counts` is given, writes this rank's send counts [ranks] into row `rank` of rank d's count matrix; then, after a
// system-scope fence (which also covers the stores of the kernels before this one in the stream, e.g. the peer
// pack), releases flag `rank` of rank d's block with `epoch`. Then thread d waits, with acquire loads and at most
// timeout_ns, until this rank's flag d reaches `epoch` (compared modulo 2^32); a wait that runs out sets this rank's
// status word to REAXMOE_ERR_DEVICE_TIMEOUT and returns. Every rank calls the signals in the same order with the
// same epochs, so when the kernel ends every peer has passed its matching signal and its earlier stores to this GPU
// are visible.
__global__ void __launch_bounds__(kMaxRanks) ep_signal_kernel(const PeerPtrs blocks, int rank, int ranks,
                                                              uint32_t epoch, const int* __restrict__ counts,
                                                              unsigned long long timeout_ns) {
  const int d = threadIdx.x;
  __threadfence_system();
  if (d < ranks) {
    uint8_t* peer = reinterpret_cast<uint8_t*>(blocks.p[d]);
    if (counts != nullptr) {
      int* row = reinterpret_cast<int*>(peer + kSigCounts) + rank * kMaxRanks;
      for (int i = 0; i < ranks; ++i) row[i] = counts[i];
    }
    uint32_t* flag = reinterpret_cast<uint32_t*>(peer + kSigFlags) + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
    uint8_t* own = reinterpret_cast<uint8_t*>(blocks.p[rank]);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(own + kSigFlags) + d;
    const uint64_t t0 = clock_ns();
    for (uint32_t n = 0;; ++n) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if ((n & 15u) == 15u && clock_ns() - t0 > timeout_ns) {
        set_status(reinterpret_cast<int*>(own + kSigStatus), REAXMOE_ERR_DEVICE_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

// Receiver: local expert ids and weights of every received record, as contiguous [n, k] arrays.
__global__ void __launch_bounds__(256) ep_unpack_meta_kernel(const uint8_t* __restrict__ records, int64_t pairs, int k,
                                                             int meta, int rec_bytes, int* __restrict__ lid,
                                                             float* __restrict__ lw) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= pairs) return;
  const int64_t rcd = i / k;
  const int j = (int)(i - rcd * k);
  const uint8_t* rec = records + rcd * rec_bytes + meta;
  lid[i] = reinterpret_cast<const int*>(rec)[j];
  lw[i] = reinterpret_cast<const float*>(rec + 4 * k)[j];
}

// Receiver permute: one CTA per segment of kSegTokens records. Phase A assigns the canonical slots of the local
// pairs (record-major inside a local expert); phase B copies each record's FP4 row and scales to its slots, the scales
// into the slot's row of the linear scale buffer (swizzle_scales_kernel then writes the 128x4 atoms the GEMM reads).
__global__ void __launch_bounds__(256) ep_permute_kernel(const uint8_t* __restrict__ records, const int* __restrict__ lid,
                                                         const int* __restrict__ seg_base, const int* __restrict__ eoff,
                                                         int n, int H, int El, int k, int rec_bytes,
                                                         uint8_t* __restrict__ rep_fp4, uint8_t* __restrict__ lin_sf,
                                                         int* __restrict__ c_map, int* __restrict__ row_token,
                                                         int* __restrict__ ga_flag) {
  __shared__ int run[kMaxExperts];
  __shared__ uint32_t mask[kMaxExperts];
  __shared__ int pos_s[kSegTokens * kMaxTopk];
  __shared__ short exp_s[kSegTokens * kMaxTopk];
  const int seg = blockIdx.x;
  const int64_t t0 = (int64_t)seg * kSegTokens;
  const int nt = (int)(kSegTokens < n - t0 ? (int64_t)kSegTokens : n - t0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < El; e += blockDim.x) {
    run[e] = eoff[e] + seg_base[(int64_t)seg * El + e];
    mask[e] = 0u;
  }
  __syncthreads();
  if (warp == 0) segment_slots(lid, t0, nt, k, El, run, mask, pos_s, exp_s, c_map);
  __syncthreads();
  if (row_token != nullptr) {
    // gather layout: the records stay where they landed; each slot records its record
    if (seg == 0 && threadIdx.x == 0) *ga_flag = 1;
    for (int i = threadIdx.x; i < nt * k; i += blockDim.x)
      if (exp_s[i] >= 0) row_token[pos_s[i]] = (int)(t0 + i / k);
    return;
  }
  const int units = H / 32;
  const int k16 = H / 16;
  const int nwarps = blockDim.x >> 5;
  constexpr int kMaxUnits = kPermUnits;
  for (int tl = warp; tl < nt; tl += nwarps) {
    const uint8_t* rec = records + (t0 + tl) * rec_bytes;
    uint4 q[kMaxUnits];
    uint16_t sb[kMaxUnits];
#pragma unroll
    for (int it = 0; it < kMaxUnits; ++it) {
      const int un = lane + 32 * it;
      if (un < units) {
        q[it] = __ldg(reinterpret_cast<const uint4*>(rec) + un);
        sb[it] = __ldg(reinterpret_cast<const unsigned short*>(rec + H / 2) + un);
      }
    }
    for (int j = 0; j < k; ++j) {
      const int e = exp_s[tl * k + j];
      if (e < 0) continue;
      const int pos = pos_s[tl * k + j];
#pragma unroll
      for (int it = 0; it < kMaxUnits; ++it) {
        const int un = lane + 32 * it;
        if (un >= units) continue;
        *reinterpret_cast<uint4*>(rep_fp4 + (int64_t)pos * (H / 2) + un * 16) = q[it];
        *reinterpret_cast<uint16_t*>(lin_sf + (int64_t)pos * k16 + un * 2) = sb[it];
      }
    }
  }
}

// Source-side combine: out[t] = bf16( sum over j in increasing order with send_map[t, j] >= 0 of
// fp32(returned[send_map[t, j]]) ), the sum started from +0. One warp per token, 8 columns per lane step; the
// compile-time-k variant issues all of a step's row loads before the arithmetic.
template <int K>
__global__ void __launch_bounds__(256) ep_combine_kernel(const __nv_bfloat16* __restrict__ ret,
                                                         const int* __restrict__ map, int m, int H, int k,
                                                         __nv_bfloat16* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int kk = K > 0 ? K : k;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < m; t += warps) {
    const int mypos = lane < kk ? map[t * kk + lane] : -1;
    int pos[K > 0 ? K : kMaxTopk];
#pragma unroll
    for (int j = 0; j < (K > 0 ? K : kMaxTopk); ++j) pos[j] = __shfl_sync(0xffffffffu, mypos, j);
    uint4* orow = reinterpret_cast<uint4*>(out + t * H);
    for (int ch = lane; ch < H / 8; ch += 32) {
      uint4 v[K > 0 ? K : kMaxTopk];
#pragma unroll
      for (int j = 0; j < (K > 0 ? K : kMaxTopk); ++j)
        v[j] = (j < kk && pos[j] >= 0) ? __ldg(reinterpret_cast<const uint4*>(ret + (int64_t)pos[j] * H) + ch)
                                       : make_uint4(0u, 0u, 0u, 0u);
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int j = 0; j < (K > 0 ? K : kMaxTopk); ++j) {
        if (j < kk && pos[j] >= 0) {
          float f[8];
          bf16x8_to_f32(v[j], f);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], f[i]);
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      orow[ch] = o;
    }
  }
}

int launch_ep_rank_ids(const int* ids, int m, int k, int E, int El, const float* a1_gscale, int* rid, int* status,
                       cudaStream_t s) {
  if (m == 0) return 0;
  ep_rank_ids_kernel<<<(unsigned)ceil_div64(m, 256), 256, 0, s>>>(ids, m, k, E, El, a1_gscale, rid, status);
  return 0;
}

int launch_ep_pack(const __nv_bfloat16* a, const float* a1_gscale, const int* ids, const float* w, const int* rid,
                   const int* seg_base, const int* roff, int m, int H, int E, int El, int k, int rec_bytes,
                   uint8_t* records, int* send_map, cudaStream_t s) {
  const int nseg = (int)ceil_div64(m, kSegTokens);
  if (nseg > 0)
    ep_pack_kernel<false><<<nseg, 256, 0, s>>>(a, a1_gscale, ids, w, rid, seg_base, roff, m, H, E, El, k, rec_bytes,
                                               records, send_map, PeerPtrs{});
  return 0;
}

int launch_ep_pack_peer(const __nv_bfloat16* a, const float* a1_gscale, const int* ids, const float* w, const int* rid,
                        const int* seg_base, const int* roff, int m, int H, int E, int El, int k, int rec_bytes,
                        const PeerPtrs& records, int* send_map, cudaStream_t s) {
  const int nseg = (int)ceil_div64(m, kSegTokens);
  if (nseg > 0)
    ep_pack_kernel<true><<<nseg, 256, 0, s>>>(a, a1_gscale, ids, w, rid, seg_base, roff, m, H, E, El, k, rec_bytes,
                                              nullptr, send_map, records);
  return 0;
}

// One thread per received record: a record with exactly one local pair is finished by the w2 epilogue (its row is
// bf16(c3 * w) rounded once, which the combine would compute too), so its slot gets the record's return address.
__global__ void __launch_bounds__(256) ep_direct_kernel(const int* __restrict__ c_map, const float* __restrict__ lw,
                                                        int n, int k, const __grid_constant__ RowRoute route, int H,
                                                        uint64_t* __restrict__ direct_dst,
                                                        float* __restrict__ direct_w) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int cnt = 0, jj = 0;
  for (int j = 0; j < k; ++j)
    if (c_map[i * k + j] >= 0) {
      ++cnt;
      jj = j;
    }
  if (cnt == 1) {
    const int slot = c_map[i * k + jj];
    direct_dst[slot] = route.row_addr(i, H);
    direct_w[slot] = lw[i * k + jj];
  } else {
    for (int j = 0; j < k; ++j) {
      const int slot = c_map[i * k + j];
      if (slot >= 0) direct_dst[slot] = 0ull;
    }
  }
}

int launch_ep_direct(const int* c_map, const float* lw, int n, int k, int H, const RowRoute& route,
                     uint64_t* direct_dst, float* direct_w, cudaStream_t s) {
  if (n > 0)
    ep_direct_kernel<<<(unsigned)ceil_div64(n, 256), 256, 0, s>>>(c_map, lw, n, k, route, H, direct_dst, direct_w);
  return 0;
}

int launch_ep_signal(const PeerPtrs& blocks, int rank, int ranks, uint32_t epoch, const int* counts,
                     unsigned long long timeout_ns, cudaStream_t s) {
  ep_signal_kernel<<<1, kMaxRanks, 0, s>>>(blocks, rank, ranks, epoch, counts, timeout_ns);
  return 0;
}

int launch_ep_unpack_meta(const uint8_t* records, int n, int k, int H, int rec_bytes, int* lid, float* lw,
                          cudaStream_t s) {
  const int64_t pairs = (int64_t)n * k;
  if (pairs == 0) return 0;
  ep_unpack_meta_kernel<<<(unsigned)ceil_div64(pairs, 256), 256, 0, s>>>(records, pairs, k, H / 2 + H / 16, rec_bytes,
                                                                          lid, lw);
  return 0;
}

int launch_ep_permute(const uint8_t* records, const int* lid, const int* seg_base, const int* eoff, int n, int H,
                      int El, int k, int rec_bytes, uint8_t* rep_fp4, uint8_t* lin_sf, int* c_map, cudaStream_t s,
                      const GatherRows* ga) {
  const int nseg = (int)ceil_div64(n, kSegTokens);
  if (nseg > 0)
    ep_permute_kernel<<<nseg, 256, 0, s>>>(records, lid, seg_base, eoff, n, H, El, k, rec_bytes, rep_fp4, lin_sf,
                                           c_map, ga ? ga->row_token : nullptr, ga ? ga->flag : nullptr);
  return 0;
}

int launch_ep_combine(const __nv_bfloat16* ret, const int* map, int m, int H, int k, __nv_bfloat16* out, int num_sms,
                      cudaStream_t s) {
  if (m == 0) return 0;
  const int64_t want = ceil_div64(m, 8), cap = (int64_t)num_sms * 8;
  const unsigned blocks = (unsigned)(want < cap ? want : cap);
  if (k == 8) ep_combine_kernel<8><<<blocks, 256, 0, s>>>(ret, map, m, H, k, out);
  else if (k == 4) ep_combine_kernel<4><<<blocks, 256, 0, s>>>(ret, map, m, H, k, out);
  else if (k == 2) ep_combine_kernel<2><<<blocks, 256, 0, s>>>(ret, map, m, H, k, out);
  else if (k == 1) ep_combine_kernel<1><<<blocks, 256, 0, s>>>(ret, map, m, H, k, out);
  else ep_combine_kernel<0><<<blocks, 256, 0, s>>>(ret, map, m, H, k, out);
  return 0;
}

}  // namespace reaxmoe
