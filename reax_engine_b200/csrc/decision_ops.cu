// decision_ops.cu -- the element-wise steps of the config-3 decision forward around the MoE block, fused so that each
// reads its inputs and writes its output once (HBM-bound). Each reproduces, at the same bf16 rounding points, the vLLM
// code it replaces:
//   rmsnorm      out = bf16(bf16(s * rsqrt(mean(s^2) + eps)) * w) [+ residual], s = bf16(a [+ b])
//                (vllm/ir/ops/layernorm.py:10-21; the sums and residual adds of Gemma4DecoderLayer.forward,
//                vllm/model_executor/models/gemma4.py:696-771, are bf16 tensor adds)
//   qkv_norm_rope  per head: RMSNorm of q and k with their learned weights, of v without (gemma4.py:512-535), then
//                NeoX rotate-half of q and k with a bf16 cos / sin table, one bf16 rounding per operation
//                (vllm/model_executor/layers/rotary_embedding/base.py forward_static)
//   gelu_tanh_mul  h = bf16(bf16(gelu_tanh(gate)) * up) (GeluAndMul native form: F.gelu(approximate="tanh") on the
//                bf16 gate, then a bf16 product; vllm/model_executor/layers/activation.py)
#include "common.cuh"
#include "kernels.cuh"

namespace reaxmoe {
namespace dops {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// bf16 add of two bf16 words (2 lanes each): fp32 sum rounded to bf16, as a torch bf16 tensor add
__device__ __forceinline__ uint32_t bf2_add(uint32_t x, uint32_t y) {
  const float lo = __uint_as_float(x << 16) + __uint_as_float(y << 16);
  const float hi = __uint_as_float(x & 0xFFFF0000u) + __uint_as_float(y & 0xFFFF0000u);
  return pack_bf16x2(lo, hi);
}

// One 128-thread CTA per row; thread i holds the 8-element pieces i, i + 128, ... (up to 4: cols <= 4096). Every input
// of the row, the residual included, is loaded before the reduction, so a row costs one memory round trip.
constexpr int RN_THREADS = 128;
constexpr int RN_PIECES = 4;

__global__ void __launch_bounds__(RN_THREADS) rmsnorm_kernel(const __nv_bfloat16* __restrict__ a,
                                                             const __nv_bfloat16* __restrict__ b,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             const __nv_bfloat16* __restrict__ res, float eps,
                                                             int cols, __nv_bfloat16* __restrict__ out) {
  __shared__ float part[RN_THREADS / 32];
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int pieces = cols >> 3;
  const uint4* pa = reinterpret_cast<const uint4*>(a + row * cols);
  const uint4* pb = b ? reinterpret_cast<const uint4*>(b + row * cols) : nullptr;
  const uint4* pr = res ? reinterpret_cast<const uint4*>(res + row * cols) : nullptr;
  uint4 s[RN_PIECES], rv[RN_PIECES];
#pragma unroll
  for (int j = 0; j < RN_PIECES; ++j) {
    const int i = tid + j * RN_THREADS;
    if (i < pieces) {
      s[j] = __ldg(pa + i);
      if (pb) {
        const uint4 u = __ldg(pb + i);
        s[j] = make_uint4(bf2_add(s[j].x, u.x), bf2_add(s[j].y, u.y), bf2_add(s[j].z, u.z), bf2_add(s[j].w, u.w));
      }
      if (pr) rv[j] = __ldg(pr + i);
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < RN_PIECES; ++j) {
    if (tid + j * RN_THREADS < pieces) {
      float f[8];
      bf16x8_to_f32(s[j], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int k = 0; k < RN_THREADS / 32; ++k) tot += part[k];
  const float r = rsqrtf(tot / (float)cols + eps);
  const uint4* pw = w ? reinterpret_cast<const uint4*>(w) : nullptr;
  uint4* po = reinterpret_cast<uint4*>(out + row * cols);
#pragma unroll
  for (int j = 0; j < RN_PIECES; ++j) {
    const int i = tid + j * RN_THREADS;
    if (i < pieces) {
      float f[8];
      bf16x8_to_f32(s[j], f);
      float wf[8];
      if (pw) bf16x8_to_f32(__ldg(pw + i), wf);
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float y0 = bf16r(f[2 * q] * r), y1 = bf16r(f[2 * q + 1] * r);
        if (pw) {
          y0 = bf16r(y0 * wf[2 * q]);        // bf16 x bf16: exact in fp32, one rounding
          y1 = bf16r(y1 * wf[2 * q + 1]);
        }
        o[q] = pack_bf16x2(y0, y1);
      }
      uint4 ov = make_uint4(o[0], o[1], o[2], o[3]);
      if (pr) ov = make_uint4(bf2_add(ov.x, rv[j].x), bf2_add(ov.y, rv[j].y), bf2_add(ov.z, rv[j].z),
                              bf2_add(ov.w, rv[j].w));
      po[i] = ov;
    }
  }
}

// rmsnorm followed by the static-scale NVFP4 quantisation of its bf16 output (the add + RMSNorm + quant fusion of
// engine/fp4_triton.py:68-90, here with vLLM's Gemma-4 norm arithmetic), for a MoE block's input: the quantiser is the
// one permute_quant applies per routed row (quant_block16_bf16 with g = 1 / gscale), so the bytes are identical to
// quantising the bf16 norm output. Thread i holds pieces i, i + 128, ...; a 16-element block is the two pieces of an
// even / odd thread pair, joined with one shuffle. Writes packed [rows, cols / 2] e2m1, linear block scales
// [rows, cols / 16] e4m3 and, when out is not null, the bf16 output too.
__global__ void __launch_bounds__(RN_THREADS) rmsnorm_nvfp4_kernel(const __nv_bfloat16* __restrict__ a,
                                                                   const __nv_bfloat16* __restrict__ b,
                                                                   const __nv_bfloat16* __restrict__ w,
                                                                   const __nv_bfloat16* __restrict__ res, float eps,
                                                                   int cols, float g, __nv_bfloat16* __restrict__ out,
                                                                   uint8_t* __restrict__ packed,
                                                                   uint8_t* __restrict__ scales) {
  __shared__ float part[RN_THREADS / 32];
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int pieces = cols >> 3;
  const uint4* pa = reinterpret_cast<const uint4*>(a + row * cols);
  const uint4* pb = b ? reinterpret_cast<const uint4*>(b + row * cols) : nullptr;
  const uint4* pr = res ? reinterpret_cast<const uint4*>(res + row * cols) : nullptr;
  uint4 s[RN_PIECES], rv[RN_PIECES];
#pragma unroll
  for (int j = 0; j < RN_PIECES; ++j) {
    const int i = tid + j * RN_THREADS;
    if (i < pieces) {
      s[j] = __ldg(pa + i);
      if (pb) {
        const uint4 u = __ldg(pb + i);
        s[j] = make_uint4(bf2_add(s[j].x, u.x), bf2_add(s[j].y, u.y), bf2_add(s[j].z, u.z), bf2_add(s[j].w, u.w));
      }
      if (pr) rv[j] = __ldg(pr + i);
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < RN_PIECES; ++j) {
    if (tid + j * RN_THREADS < pieces) {
      float f[8];
      bf16x8_to_f32(s[j], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int k = 0; k < RN_THREADS / 32; ++k) tot += part[k];
  const float r = rsqrtf(tot / (float)cols + eps);
  const uint4* pw = w ? reinterpret_cast<const uint4*>(w) : nullptr;
#pragma unroll
  for (int j = 0; j < RN_PIECES; ++j) {
    const int i = tid + j * RN_THREADS;
    const bool live = i < pieces;            // pieces is a multiple of 32: both threads of a pair agree
    uint4 ov = make_uint4(0u, 0u, 0u, 0u);
    if (live) {
      float f[8];
      bf16x8_to_f32(s[j], f);
      float wf[8];
      if (pw) bf16x8_to_f32(__ldg(pw + i), wf);
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float y0 = bf16r(f[2 * q] * r), y1 = bf16r(f[2 * q + 1] * r);
        if (pw) {
          y0 = bf16r(y0 * wf[2 * q]);
          y1 = bf16r(y1 * wf[2 * q + 1]);
        }
        o[q] = pack_bf16x2(y0, y1);
      }
      ov = make_uint4(o[0], o[1], o[2], o[3]);
      if (pr) ov = make_uint4(bf2_add(ov.x, rv[j].x), bf2_add(ov.y, rv[j].y), bf2_add(ov.z, rv[j].z),
                              bf2_add(ov.w, rv[j].w));
      if (out) reinterpret_cast<uint4*>(out + row * cols)[i] = ov;
    }
    // the odd thread's piece completes the even thread's 16-element block
    const uint32_t n0 = __shfl_xor_sync(0xffffffffu, ov.x, 1), n1 = __shfl_xor_sync(0xffffffffu, ov.y, 1);
    const uint32_t n2 = __shfl_xor_sync(0xffffffffu, ov.z, 1), n3 = __shfl_xor_sync(0xffffffffu, ov.w, 1);
    if (live && (tid & 1) == 0) {
      const uint32_t xw[8] = {ov.x, ov.y, ov.z, ov.w, n0, n1, n2, n3};
      uint32_t lo, hi;
      const uint32_t sb = quant_block16_bf16(xw, g, lo, hi);
      const int blk = i >> 1;
      *reinterpret_cast<uint2*>(packed + row * (cols / 2) + blk * 8) = make_uint2(lo, hi);
      scales[row * (cols / 16) + blk] = (uint8_t)sb;
    }
  }
}

// PER consecutive bf16 <-> floats with one vector access (PER = 2, 4 or 8; the address is PER*2-byte aligned)
template <int PER>
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, float* f) {
  uint32_t w[PER / 2];
  if constexpr (PER == 8) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (PER == 4) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  }
#pragma unroll
  for (int i = 0; i < PER / 2; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <int PER>
__device__ __forceinline__ void store_bf16(__nv_bfloat16* p, const float* f) {
  uint32_t w[PER / 2];
#pragma unroll
  for (int i = 0; i < PER / 2; ++i) w[i] = pack_bf16x2(f[2 * i], f[2 * i + 1]);
  if constexpr (PER == 8) {
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if constexpr (PER == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  }
}

// Grid (token, group of 32 heads): 8 warps, each taking 4 heads whose rows it loads up front as raw words, then
// normalises and rotates them one by one. Lane l holds the rotation pairs themselves -- elements
// [l * D/64, (l + 1) * D/64) of each half of the head -- so the rotate-half needs no exchange between lanes and
// the only shuffles are the 5 of the row reduction (shuffles go through the MIO pipe, which a per-pair exchange
// saturated). D = 64, 128 or 256.
constexpr int QKV_WARPS = 8;
constexpr int QKV_HPW = 4;                 // heads per warp
constexpr int QKV_HEADS_PER_CTA = QKV_WARPS * QKV_HPW;

template <int N>
__device__ __forceinline__ void load_raw_bf16(const __nv_bfloat16* p, uint32_t (&w)[(N + 1) / 2]) {
  if constexpr (N == 4) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (N == 2) {
    w[0] = __ldg(reinterpret_cast<const uint32_t*>(p));
  } else {
    w[0] = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p));
  }
}
template <int N>
__device__ __forceinline__ void unpack_bf16(const uint32_t (&w)[(N + 1) / 2], float* f) {
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = __uint_as_float((i & 1) ? (w[i / 2] & 0xFFFF0000u) : (w[i / 2] << 16));
}
template <int N>
__device__ __forceinline__ void store_half(__nv_bfloat16* p, const float* f) {
  if constexpr (N == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]));
  } else if constexpr (N == 2) {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(f[0], f[1]);
  } else {
    *p = __float2bfloat16_rn(f[0]);
  }
}

template <int D>
__global__ void __launch_bounds__(QKV_WARPS * 32) qkv_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                                       const __nv_bfloat16* __restrict__ qw,
                                                                       const __nv_bfloat16* __restrict__ kw,
                                                                       const __nv_bfloat16* __restrict__ cos_t,
                                                                       const __nv_bfloat16* __restrict__ sin_t,
                                                                       const int64_t* __restrict__ pos, float eps,
                                                                       int hq, int hk, __nv_bfloat16* __restrict__ q,
                                                                       __nv_bfloat16* __restrict__ k,
                                                                       __nv_bfloat16* __restrict__ v) {
  constexpr int H2 = D / 64;                         // elements per lane in each half
  constexpr int NW = (H2 + 1) / 2;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int heads = hq + 2 * hk;
  const int64_t t = blockIdx.x;
  const int hbase = blockIdx.y * QKV_HEADS_PER_CTA + warp;     // heads hbase, hbase + 8, ...
  const int e0 = lane * H2;                          // this lane's first element in each half
  uint32_t r1[QKV_HPW][NW], r2[QKV_HPW][NW];
#pragma unroll
  for (int i = 0; i < QKV_HPW; ++i) {
    const int h = hbase + i * QKV_WARPS;
    if (h < heads) {
      const __nv_bfloat16* src = qkv + t * (int64_t)heads * D + (int64_t)h * D;
      load_raw_bf16<H2>(src + e0, r1[i]);
      load_raw_bf16<H2>(src + D / 2 + e0, r2[i]);
    }
  }
  const int64_t p = pos[t];
#pragma unroll
  for (int i = 0; i < QKV_HPW; ++i) {
    const int h = hbase + i * QKV_WARPS;
    if (h < heads) {                                 // uniform across the warp
      float x1[H2], x2[H2];
      unpack_bf16<H2>(r1[i], x1);
      unpack_bf16<H2>(r2[i], x2);
      float ss = 0.0f;
#pragma unroll
      for (int e = 0; e < H2; ++e) ss = fmaf(x1[e], x1[e], fmaf(x2[e], x2[e], ss));
      const float r = rsqrtf(warp_sum(ss) / (float)D + eps);
      const bool is_q = h < hq, is_k = !is_q && h < hq + hk;
      const __nv_bfloat16* wt = is_q ? qw : (is_k ? kw : nullptr);
#pragma unroll
      for (int e = 0; e < H2; ++e) {
        x1[e] = bf16r(x1[e] * r);
        x2[e] = bf16r(x2[e] * r);
      }
      __nv_bfloat16* dst;
      if (is_q) {
        dst = q + (t * hq + h) * (int64_t)D;
      } else if (is_k) {
        dst = k + (t * hk + (h - hq)) * (int64_t)D;
      } else {
        dst = v + (t * hk + (h - hq - hk)) * (int64_t)D;
      }
      if (wt) {
        uint32_t w1[NW], w2[NW], cw[NW], sw[NW];
        load_raw_bf16<H2>(wt + e0, w1);
        load_raw_bf16<H2>(wt + D / 2 + e0, w2);
        load_raw_bf16<H2>(cos_t + p * (D / 2) + e0, cw);
        load_raw_bf16<H2>(sin_t + p * (D / 2) + e0, sw);
        float wf1[H2], wf2[H2], cs[H2], sn[H2];
        unpack_bf16<H2>(w1, wf1);
        unpack_bf16<H2>(w2, wf2);
        unpack_bf16<H2>(cw, cs);
        unpack_bf16<H2>(sw, sn);
#pragma unroll
        for (int e = 0; e < H2; ++e) {
          const float a = bf16r(x1[e] * wf1[e]), b = bf16r(x2[e] * wf2[e]);
          // x1' = x1 cos - x2 sin, x2' = x2 cos + x1 sin -- each product and the sum rounded to bf16
          x1[e] = bf16r(bf16r(a * cs[e]) - bf16r(b * sn[e]));
          x2[e] = bf16r(bf16r(b * cs[e]) + bf16r(a * sn[e]));
        }
      }
      store_half<H2>(dst + e0, x1);
      store_half<H2>(dst + D / 2 + e0, x2);
    }
  }
}

// gate = gu[:, :I], up = gu[:, I:]; 8 columns per thread.
__global__ void __launch_bounds__(256) gelu_tanh_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t rows,
                                                            int inter, __nv_bfloat16* __restrict__ h) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = inter >> 3;
  if (i >= rows * per_row) return;
  const int64_t row = i / per_row;
  const int c = (int)(i - row * per_row);
  const uint4 g = __ldg(reinterpret_cast<const uint4*>(gu + row * 2 * inter) + c);
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(gu + row * 2 * inter + inter) + c);
  float gf[8], uf[8];
  bf16x8_to_f32(g, gf);
  bf16x8_to_f32(u, uf);
  const float kBeta = 0.7978845608028654f;          // sqrt(2 / pi)
  const float kKappa = 0.044715f;
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float y[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float x = gf[2 * j + e];
      const float inner = kBeta * (x + kKappa * (x * x * x));
      const float act = bf16r(0.5f * x * (1.0f + tanhf(inner)));
      y[e] = act * uf[2 * j + e];
    }
    o[j] = pack_bf16x2(y[0], y[1]);
  }
  reinterpret_cast<uint4*>(h + row * inter)[c] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace dops

int launch_rmsnorm(const void* a, const void* b, const void* w, const void* res, float eps, int64_t rows, int cols,
                   void* out, cudaStream_t s) {
  if (rows == 0) return 0;
  if (rows > 0x7FFFFFFFLL) return REAXMOE_ERR_BAD_SHAPE;
  dops::rmsnorm_kernel<<<(unsigned)rows, dops::RN_THREADS, 0, s>>>(
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
      static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(res), eps, cols,
      static_cast<__nv_bfloat16*>(out));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : REAXMOE_ERR_CUDA;
}

int launch_rmsnorm_nvfp4(const void* a, const void* b, const void* w, const void* res, float eps, int64_t rows,
                         int cols, float gscale, void* out, uint8_t* packed, uint8_t* scales, cudaStream_t s) {
  if (rows == 0) return 0;
  if (rows > 0x7FFFFFFFLL) return REAXMOE_ERR_BAD_SHAPE;
  dops::rmsnorm_nvfp4_kernel<<<(unsigned)rows, dops::RN_THREADS, 0, s>>>(
      static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b),
      static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(res), eps, cols,
      1.0f / gscale, static_cast<__nv_bfloat16*>(out), packed, scales);   // IEEE division, as permute_quant
  return cudaPeekAtLastError() == cudaSuccess ? 0 : REAXMOE_ERR_CUDA;
}

int launch_qkv_norm_rope(const void* qkv, const void* qw, const void* kw, const void* cos_t, const void* sin_t,
                         const int64_t* pos, float eps, int64_t n, int hq, int hk, int d, void* q, void* k, void* v,
                         cudaStream_t s) {
  if (n == 0) return 0;
  if (n > 0x7FFFFFFFLL) return REAXMOE_ERR_BAD_SHAPE;
  const dim3 grid((unsigned)n, (unsigned)((hq + 2 * hk + dops::QKV_HEADS_PER_CTA - 1) / dops::QKV_HEADS_PER_CTA));
#define REAXMOE_QKV(DD)                                                                                          \
  dops::qkv_norm_rope_kernel<DD><<<grid, dops::QKV_WARPS * 32, 0, s>>>(                                          \
      static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(qw),                            \
      static_cast<const __nv_bfloat16*>(kw), static_cast<const __nv_bfloat16*>(cos_t),                          \
      static_cast<const __nv_bfloat16*>(sin_t), pos, eps, hq, hk, static_cast<__nv_bfloat16*>(q),                \
      static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v))
  switch (d) {
    case 64: REAXMOE_QKV(64); break;
    case 128: REAXMOE_QKV(128); break;
    case 256: REAXMOE_QKV(256); break;
    default: return REAXMOE_ERR_UNSUPPORTED;
  }
#undef REAXMOE_QKV
  return cudaPeekAtLastError() == cudaSuccess ? 0 : REAXMOE_ERR_CUDA;
}

int launch_gelu_tanh_mul(const void* gu, int64_t rows, int inter, void* h, cudaStream_t s) {
  const int64_t items = rows * (inter / 8);
  if (items == 0) return 0;
  dops::gelu_tanh_mul_kernel<<<(unsigned)ceil_div64(items, 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(gu), rows, inter, static_cast<__nv_bfloat16*>(h));
  return cudaPeekAtLastError() == cudaSuccess ? 0 : REAXMOE_ERR_CUDA;
}

}  // namespace reaxmoe
