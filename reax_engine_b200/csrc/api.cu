// api.cu -- the extern "C" entry points of include/reaxmoe.h: argument checks, workspace layout and the
// launch sequence of the layer. No allocation, no host synchronisation on the forward path.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

namespace reaxmoe {

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int set_error(int code, const char* msg) { return fail(code, "%s", msg); }

static int cuda_check(const char* what) {
  const cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return fail(REAXMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return 0;
}

static int g_sm_budget = 0;   // 0: every SM (reaxmoe_set_sm_budget)

static int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  return (g_sm_budget > 0 && g_sm_budget < n) ? g_sm_budget : n;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// local_topk: an expert-parallel receiver's problem, whose records may carry more pairs (topk) than it owns
// experts; only the local pairs are used.
static int check_problem(const reaxmoe_problem* p, bool local_topk = false) {
  if (p == nullptr) return fail(REAXMOE_ERR_NULL, "problem is NULL");
  if (p->experts < 1 || p->experts > kMaxExperts)
    return fail(REAXMOE_ERR_TOO_MANY_EXPERTS, "experts=%d outside [1, %d]", p->experts, kMaxExperts);
  if (p->topk < 1 || p->topk > kMaxTopk || (!local_topk && p->topk > p->experts))
    return fail(REAXMOE_ERR_TOO_MANY_EXPERTS, "topk=%d outside [1, min(%d, experts)]", p->topk, kMaxTopk);
  if (p->hidden < 256 || p->hidden > 3072 || p->hidden % 128 != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "hidden=%d must be a multiple of 128 in [256, 3072]", p->hidden);
  if (p->inter < 256 || p->inter > 3072 || p->inter % 64 != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "inter=%d must be a multiple of 64 in [256, 3072]", p->inter);
  if (p->tokens < 0) return fail(REAXMOE_ERR_BAD_SHAPE, "tokens=%d < 0", p->tokens);
  if ((int64_t)p->tokens * p->topk > (int64_t)1 << 30)
    return fail(REAXMOE_ERR_BAD_SHAPE, "tokens*topk=%lld too large", (long long)p->tokens * p->topk);
  if (p->activation != REAXMOE_ACT_SILU && p->activation != REAXMOE_ACT_GELU_TANH)
    return fail(REAXMOE_ERR_BAD_SHAPE, "activation=%d unknown", p->activation);
  return 0;
}

// The shape checks of every entry point, for the other translation units (reaxmoe_plan_static).
int check_problem_shape(const reaxmoe_problem* p) { return check_problem(p); }

// Workspace regions, each 256-byte aligned.
struct Layout {
  size_t status, seg_counts, seg_base, counts, eoff, boff, tile_prefix, c_map, rep_fp4, lin_sf, rep_sf, int_fp4,
      int_sf, c3, tok_fp4, tok_sf, row_token, ga_flag, total;
};

static size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

static Layout layout(const reaxmoe_problem* p) {
  Layout L;
  const int64_t m = p->tokens, k = p->topk, E = p->experts, H = p->hidden, I = p->inter;
  const int64_t slots = m * k;
  const int64_t nseg = ceil_div64(m, kSegTokens);
  const int64_t sfblk = sf_row_blocks(slots, (int)E);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = up256(off + bytes);
    return o;
  };
  L.status = take(64);
  L.seg_counts = take((size_t)nseg * E * 4);
  L.seg_base = take((size_t)nseg * E * 4);
  L.counts = take((size_t)E * 4);
  L.eoff = take((size_t)(E + 1) * 4);
  L.boff = take((size_t)(E + 1) * 4);
  L.tile_prefix = take((size_t)(E + 1) * 4);
  L.c_map = take((size_t)slots * 4);
  L.rep_fp4 = take((size_t)slots * (H / 2));
  L.lin_sf = take((size_t)slots * (H / 16));
  L.rep_sf = take((size_t)sfblk * (H / 64) * 512);
  L.int_fp4 = take((size_t)slots * (I / 2));
  L.int_sf = take((size_t)sfblk * (I / 64) * 512);
  L.c3 = take((size_t)slots * H * 2);
  L.tok_fp4 = take((size_t)m * (H / 2));
  L.tok_sf = take((size_t)m * (H / 16));
  L.row_token = take((size_t)slots * 4);
  L.ga_flag = take(64);
  L.total = off;
  return L;
}

struct WS {
  int* status;
  int* seg_counts;
  int* seg_base;
  int* counts;
  int* eoff;
  int* boff;
  int* tile_prefix;
  int* c_map;
  uint8_t* rep_fp4;
  uint8_t* lin_sf;  // scale bytes of the routed rows in slot order, [slots, H/16] (permute -> swizzle)
  uint8_t* rep_sf;
  uint8_t* int_fp4;
  uint8_t* int_sf;
  __nv_bfloat16* c3;
  GatherRows ga;    // the gather layout of the w13 A operand (token-major rows, slot -> token map, layout flag)
};

static WS carve(void* ws, const Layout& L) {
  uint8_t* b = static_cast<uint8_t*>(ws);
  WS w;
  w.status = reinterpret_cast<int*>(b + L.status);
  w.seg_counts = reinterpret_cast<int*>(b + L.seg_counts);
  w.seg_base = reinterpret_cast<int*>(b + L.seg_base);
  w.counts = reinterpret_cast<int*>(b + L.counts);
  w.eoff = reinterpret_cast<int*>(b + L.eoff);
  w.boff = reinterpret_cast<int*>(b + L.boff);
  w.tile_prefix = reinterpret_cast<int*>(b + L.tile_prefix);
  w.c_map = reinterpret_cast<int*>(b + L.c_map);
  w.rep_fp4 = b + L.rep_fp4;
  w.lin_sf = b + L.lin_sf;
  w.rep_sf = b + L.rep_sf;
  w.int_fp4 = b + L.int_fp4;
  w.int_sf = b + L.int_sf;
  w.c3 = reinterpret_cast<__nv_bfloat16*>(b + L.c3);
  w.ga.tok_fp4 = b + L.tok_fp4;
  w.ga.tok_sf = b + L.tok_sf;
  w.ga.row_token = reinterpret_cast<int*>(b + L.row_token);
  w.ga.flag = reinterpret_cast<int*>(b + L.ga_flag);
  return w;
}

static int check_ws(const reaxmoe_problem* p, void* ws, size_t bytes, Layout* L) {
  *L = layout(p);
  if (ws == nullptr) return fail(REAXMOE_ERR_WORKSPACE, "workspace is NULL");
  if (!aligned16(ws)) return fail(REAXMOE_ERR_MISALIGNED, "workspace not 16-byte aligned");
  if (bytes < L->total)
    return fail(REAXMOE_ERR_WORKSPACE, "workspace %zu bytes < required %zu", bytes, L->total);
  return 0;
}

// Expert-parallel dispatch workspace: rank ids of the pairs and the routing data over ranks.
struct EpDispatchLayout {
  size_t status, rid, seg_counts, seg_base, roff, boff, tile_prefix, total;
};

static EpDispatchLayout ep_dispatch_layout(const reaxmoe_problem* p, int ranks) {
  EpDispatchLayout L;
  const int64_t m = p->tokens, k = p->topk;
  const int64_t nseg = ceil_div64(m, kSegTokens);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = up256(off + bytes);
    return o;
  };
  L.status = take(64);
  L.rid = take((size_t)m * k * 4);
  L.seg_counts = take((size_t)nseg * ranks * 4);
  L.seg_base = take((size_t)nseg * ranks * 4);
  L.roff = take((size_t)(ranks + 1) * 4);
  L.boff = take((size_t)(ranks + 1) * 4);
  L.tile_prefix = take((size_t)(ranks + 1) * 4);
  L.total = off;
  return L;
}

static int check_ep(const reaxmoe_problem* p, int ranks) {
  int rc = check_problem(p);
  if (rc) return rc;
  if (ranks < 1 || ranks > kMaxRanks || p->experts % ranks != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "ranks=%d must be in [1, %d] and divide experts=%d", ranks, kMaxRanks,
                p->experts);
  return 0;
}

// Expert-parallel receiver workspace: the single-GPU layout of the local problem, then the records' local ids and
// weights as [tokens, topk] arrays, then (peer transport) the direct-row table per slot: return address and weight.
static size_t ep_expert_lid(const Layout& L) { return L.total; }
static size_t ep_expert_lw(const reaxmoe_problem* p, const Layout& L) {
  return up256(L.total + (size_t)p->tokens * p->topk * 4);
}
static size_t ep_expert_direct(const reaxmoe_problem* p, const Layout& L) {
  return up256(ep_expert_lw(p, L) + (size_t)p->tokens * p->topk * 4);
}
static size_t ep_expert_direct_w(const reaxmoe_problem* p, const Layout& L) {
  return up256(ep_expert_direct(p, L) + (size_t)p->tokens * p->topk * 8);
}
static size_t ep_expert_total(const reaxmoe_problem* p, const Layout& L) {
  return up256(ep_expert_direct_w(p, L) + (size_t)p->tokens * p->topk * 4);
}

// REAXMOE_EP_DIRECT_ROWS=1 turns on the w2-epilogue direct rows of the peer transport: a record with one local pair
// gets its row stored to its source rank by the w2 epilogue instead of the pre-sum kernel (bit-identical rows). Off
// by default: on 2 B200s the epilogue's peer stores slowed the w2 GEMM more than the pre-sum pass they save (26.7M
// against 30.1M tokens/s at 65,536 tokens per rank). Read once per process.
static bool ep_direct_rows() {
  static const bool on = [] {
    const char* v = getenv("REAXMOE_EP_DIRECT_ROWS");
    return v != nullptr && v[0] == '1';
  }();
  return on;
}

static unsigned long long device_timeout_ns() {
  const char* s = getenv("REAXMOE_WAIT_TIMEOUT_NS");
  if (s != nullptr && *s) return strtoull(s, nullptr, 10);
  return 4000000000ull;  // 4 s: far above any legitimate intra-CTA wait
}

static int do_plan(const reaxmoe_problem* p, const int32_t* ids, const WS& w, int32_t* ps1, int32_t* ps2,
                   cudaStream_t s) {
  const int nseg = (int)ceil_div64(p->tokens, kSegTokens);
  cudaMemsetAsync(w.status, 0, sizeof(int), s);
  launch_count(ids, p->tokens, p->topk, p->experts, w.seg_counts, w.status, s);
  launch_plan(w.seg_counts, nseg, p->experts, w.seg_base, w.counts, w.eoff, w.boff, w.tile_prefix, ps1, ps2,
              2 * p->inter, p->hidden, p->hidden, p->inter, s);
  return cuda_check("plan");
}

static GemmLaunch w13_launch(const reaxmoe_problem* p, const WS& w, const void* rep_fp4, const void* rep_sf,
                             const void* w1, const void* w1_sf, const float* alphas, const float* a2_gscale,
                             void* int_fp4, void* int_sf) {
  GemmLaunch g;
  memset(&g, 0, sizeof(g));
  g.mode = 1;
  g.act = p->activation;
  g.a = rep_fp4;
  g.slots = (int64_t)p->tokens * p->topk;
  g.a_sf = rep_sf;
  g.b = w1;
  g.b_sf = w1_sf;
  g.alphas = alphas;
  g.E = p->experts;
  g.N = 2 * p->inter;
  g.K = p->hidden;
  g.counts = w.counts;
  g.eoff = w.eoff;
  g.boff = w.boff;
  g.tile_prefix = w.tile_prefix;
  g.q_out = int_fp4;
  g.q_sf = int_sf;
  g.q_gscale = a2_gscale;
  g.status = w.status;
  g.timeout_ns = device_timeout_ns();
  return g;
}

// The w13 launch of the gather layout: A rows through the workspace's slot -> token map, from tok (token-major
// [tokens, hidden/2]) when the permute stage wrote that layout, else from the per-slot rows rep.
static GemmLaunch w13_gather_launch(const reaxmoe_problem* p, const WS& w, const void* tok, const void* rep,
                                    const void* rep_sf, const void* w1, const void* w1_sf, const float* alphas,
                                    const float* a2_gscale, void* int_fp4, void* int_sf) {
  GemmLaunch g = w13_launch(p, w, rep, rep_sf, w1, w1_sf, alphas, a2_gscale, int_fp4, int_sf);
  g.a_tok = tok;
  g.row_token = w.ga.row_token;
  g.ga_flag = w.ga.flag;
  g.tokens = p->tokens;
  return g;
}

static GemmLaunch w2_launch(const reaxmoe_problem* p, const WS& w, const void* int_fp4, const void* int_sf,
                            const void* w2, const void* w2_sf, const float* alphas, void* c3) {
  GemmLaunch g;
  memset(&g, 0, sizeof(g));
  g.mode = 0;
  g.a = int_fp4;
  g.slots = (int64_t)p->tokens * p->topk;
  g.a_sf = int_sf;
  g.b = w2;
  g.b_sf = w2_sf;
  g.alphas = alphas;
  g.E = p->experts;
  g.N = p->hidden;
  g.K = p->inter;
  g.counts = w.counts;
  g.eoff = w.eoff;
  g.boff = w.boff;
  g.tile_prefix = w.tile_prefix;
  g.out = c3;
  g.status = w.status;
  g.timeout_ns = device_timeout_ns();
  return g;
}

}  // namespace reaxmoe

using namespace reaxmoe;

extern "C" {

int32_t reaxmoe_version(void) { return 100; }

size_t reaxmoe_last_error(char* buf, size_t len) {
  if (buf != nullptr && len > 0) {
    const size_t n = g_last_error.size() < len - 1 ? g_last_error.size() : len - 1;
    memcpy(buf, g_last_error.data(), n);
    buf[n] = '\0';
  }
  return g_last_error.size();
}

size_t reaxmoe_workspace_size(const reaxmoe_problem* p) {
  if (check_problem(p)) return 0;
  return layout(p).total;
}

int reaxmoe_route(const float* logits, const float* per_expert_scale, int32_t tokens, int32_t experts, int32_t topk,
                  int32_t* topk_ids, float* topk_weights, void* stream) {
  if (experts < 1 || experts > kMaxExperts || topk < 1 || topk > kMaxTopk || topk > experts)
    return fail(REAXMOE_ERR_TOO_MANY_EXPERTS, "route: experts=%d topk=%d unsupported", experts, topk);
  if (tokens < 0) return fail(REAXMOE_ERR_BAD_SHAPE, "route: tokens=%d < 0", tokens);
  if (tokens == 0) return 0;
  if (logits == nullptr || topk_ids == nullptr || topk_weights == nullptr)
    return fail(REAXMOE_ERR_NULL, "route: NULL pointer");
  launch_route(logits, per_expert_scale, tokens, experts, topk, topk_ids, topk_weights,
               static_cast<cudaStream_t>(stream));
  return cuda_check("route");
}

void reaxmoe_set_sm_budget(int32_t sms) { g_sm_budget = sms > 0 ? sms : 0; }

int reaxmoe_router_topk(const void* hidden_states, const void* router_scale, const void* router_weight,
                        const float* per_expert_scale, float eps, int32_t tokens, int32_t hidden, int32_t experts,
                        int32_t topk, int32_t* topk_ids, float* topk_weights, float* logits, int32_t* status,
                        void* stream) {
  if (experts != 32 && experts != 64 && experts != 128)
    return fail(REAXMOE_ERR_UNSUPPORTED, "router_topk: experts=%d (32, 64 or 128)", experts);
  if (topk < 1 || topk > kMaxTopk || topk > experts)
    return fail(REAXMOE_ERR_TOO_MANY_EXPERTS, "router_topk: topk=%d outside [1, min(%d, experts)]", topk, kMaxTopk);
  if (hidden < 128 || hidden > 3072 || hidden % 128 != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "router_topk: hidden=%d must be a multiple of 128 in [128, 3072]", hidden);
  if (tokens < 0) return fail(REAXMOE_ERR_BAD_SHAPE, "router_topk: tokens=%d < 0", tokens);
  if (tokens == 0) return 0;
  if (!hidden_states || !router_scale || !router_weight || !topk_ids || !topk_weights)
    return fail(REAXMOE_ERR_NULL, "router_topk: NULL pointer");
  if (!aligned16(hidden_states) || !aligned16(router_weight) || (logits != nullptr && !aligned16(logits)))
    return fail(REAXMOE_ERR_MISALIGNED, "router_topk: hidden_states, router_weight and logits must be 16-byte aligned");
  RouterLaunch r;
  memset(&r, 0, sizeof(r));
  r.x = hidden_states;
  r.scale = router_scale;
  r.w = router_weight;
  r.pes = per_expert_scale;
  // the reference multiplies by root_size.to(bf16), root_size = torch.tensor(hidden**-0.5) (fp32)
  r.root = __bfloat162float(__float2bfloat16_rn((float)(1.0 / sqrt((double)hidden))));
  r.eps = eps;
  r.T = tokens;
  r.H = hidden;
  r.E = experts;
  r.K = topk;
  r.ids = topk_ids;
  r.wts = topk_weights;
  r.logits = logits;
  r.status = status;
  r.timeout_ns = device_timeout_ns();
  r.num_sms = num_sms();
  const int rc = launch_router_topk(r, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "router_topk launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("router_topk");
}

int reaxmoe_rmsnorm(const void* a, const void* b, const void* weight, const void* residual, float eps, int64_t rows,
                    int32_t cols, void* out, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 256 != 0 || cols > 4096)
    return fail(REAXMOE_ERR_BAD_SHAPE, "rmsnorm: rows=%lld cols=%d (cols a multiple of 256, <= 4096)",
                (long long)rows, cols);
  if (rows == 0) return 0;
  if (!a || !out) return fail(REAXMOE_ERR_NULL, "rmsnorm: NULL input or output");
  if (!aligned16(a) || !aligned16(out) || (b && !aligned16(b)) || (weight && !aligned16(weight)) ||
      (residual && !aligned16(residual)))
    return fail(REAXMOE_ERR_MISALIGNED, "rmsnorm: tensors must be 16-byte aligned");
  const int rc = launch_rmsnorm(a, b, weight, residual, eps, rows, cols, out, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "rmsnorm launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("rmsnorm");
}

int reaxmoe_rmsnorm_nvfp4(const void* a, const void* b, const void* weight, const void* residual, float eps,
                          int64_t rows, int32_t cols, float gscale, void* out, void* packed, void* scales,
                          void* stream) {
  if (rows < 0 || cols <= 0 || cols % 256 != 0 || cols > 4096)
    return fail(REAXMOE_ERR_BAD_SHAPE, "rmsnorm_nvfp4: rows=%lld cols=%d (cols a multiple of 256, <= 4096)",
                (long long)rows, cols);
  if (!(gscale > 0.0f)) return fail(REAXMOE_ERR_BAD_SHAPE, "rmsnorm_nvfp4: gscale must be > 0");
  if (rows == 0) return 0;
  if (!a || !packed || !scales) return fail(REAXMOE_ERR_NULL, "rmsnorm_nvfp4: NULL input or output");
  if (!aligned16(a) || !aligned16(packed) || !aligned16(scales) || (out && !aligned16(out)) || (b && !aligned16(b)) ||
      (weight && !aligned16(weight)) || (residual && !aligned16(residual)))
    return fail(REAXMOE_ERR_MISALIGNED, "rmsnorm_nvfp4: tensors must be 16-byte aligned");
  const int rc = launch_rmsnorm_nvfp4(a, b, weight, residual, eps, rows, cols, gscale, out,
                                      static_cast<uint8_t*>(packed), static_cast<uint8_t*>(scales),
                                      static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "rmsnorm_nvfp4 launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("rmsnorm_nvfp4");
}

int reaxmoe_qkv_norm_rope(const void* qkv, const void* q_weight, const void* k_weight, const void* cos_table,
                          const void* sin_table, const int64_t* positions, float eps, int64_t tokens, int32_t q_heads,
                          int32_t kv_heads, int32_t head_dim, void* q, void* k, void* v, void* stream) {
  if (tokens < 0 || q_heads <= 0 || kv_heads <= 0 || (head_dim != 64 && head_dim != 128 && head_dim != 256))
    return fail(REAXMOE_ERR_BAD_SHAPE, "qkv_norm_rope: tokens=%lld heads=%d/%d head_dim=%d (64, 128 or 256)",
                (long long)tokens, q_heads, kv_heads, head_dim);
  if (tokens == 0) return 0;
  if (!qkv || !q_weight || !k_weight || !cos_table || !sin_table || !positions || !q || !k || !v)
    return fail(REAXMOE_ERR_NULL, "qkv_norm_rope: NULL pointer");
  const int rc = launch_qkv_norm_rope(qkv, q_weight, k_weight, cos_table, sin_table, positions, eps, tokens, q_heads,
                                      kv_heads, head_dim, q, k, v, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "qkv_norm_rope launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("qkv_norm_rope");
}

int reaxmoe_gelu_tanh_mul(const void* gate_up, int64_t rows, int32_t inter, void* out, void* stream) {
  if (rows < 0 || inter <= 0 || inter % 8 != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "gelu_tanh_mul: rows=%lld inter=%d (a multiple of 8)", (long long)rows, inter);
  if (rows == 0) return 0;
  if (!gate_up || !out) return fail(REAXMOE_ERR_NULL, "gelu_tanh_mul: NULL pointer");
  if (!aligned16(gate_up) || !aligned16(out))
    return fail(REAXMOE_ERR_MISALIGNED, "gelu_tanh_mul: tensors must be 16-byte aligned");
  const int rc = launch_gelu_tanh_mul(gate_up, rows, inter, out, static_cast<cudaStream_t>(stream));
  if (rc) return fail(rc, "gelu_tanh_mul launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("gelu_tanh_mul");
}

int reaxmoe_plan(const reaxmoe_problem* p, const int32_t* topk_ids, void* workspace, size_t workspace_bytes,
                 int32_t* expert_offsets, int32_t* blockscale_offsets, int32_t* problem_sizes1,
                 int32_t* problem_sizes2, void* stream) {
  int rc = check_problem(p);
  if (rc) return rc;
  Layout L;
  if ((rc = check_ws(p, workspace, workspace_bytes, &L))) return rc;
  // zero tokens still write the outputs: offsets of 0 and problem sizes (0, n, k)
  if (p->tokens > 0 && topk_ids == nullptr) return fail(REAXMOE_ERR_NULL, "plan: topk_ids is NULL");
  const WS w = carve(workspace, L);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = do_plan(p, topk_ids, w, problem_sizes1, problem_sizes2, s))) return rc;
  const size_t n = (size_t)(p->experts + 1) * 4;
  if (expert_offsets != nullptr) cudaMemcpyAsync(expert_offsets, w.eoff, n, cudaMemcpyDefault, s);
  if (blockscale_offsets != nullptr) cudaMemcpyAsync(blockscale_offsets, w.boff, n, cudaMemcpyDefault, s);
  return cuda_check("plan copy-out");
}

int reaxmoe_permute_quant(const reaxmoe_problem* p, const void* a, const float* a1_gscale, const int32_t* topk_ids,
                          void* workspace, size_t workspace_bytes, void* rep_fp4, void* rep_sf, int32_t* c_map,
                          void* stream) {
  int rc = check_problem(p);
  if (rc) return rc;
  Layout L;
  if ((rc = check_ws(p, workspace, workspace_bytes, &L))) return rc;
  if (p->tokens == 0) return 0;
  if (!a || !a1_gscale || !topk_ids || !rep_sf || !c_map)
    return fail(REAXMOE_ERR_NULL, "permute_quant: NULL pointer");
  if (!aligned16(a) || !aligned16(rep_fp4) || !aligned16(rep_sf))
    return fail(REAXMOE_ERR_MISALIGNED, "permute_quant: a, rep_fp4 and rep_sf must be 16-byte aligned");
  const WS w = carve(workspace, L);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rep_fp4 == nullptr) {
    // gather layout, kept in the workspace for reaxmoe_gemm_w13 with rep_fp4 == NULL
    launch_permute_quant(static_cast<const __nv_bfloat16*>(a), a1_gscale, topk_ids, w.seg_base, w.eoff, w.boff,
                         p->tokens, p->hidden, p->experts, p->topk, w.rep_fp4, w.lin_sf, c_map, s, &w.ga);
    launch_swizzle_scales(w.lin_sf, w.tile_prefix, w.counts, w.eoff, p->experts, p->hidden,
                          (int64_t)p->tokens * p->topk, static_cast<uint8_t*>(rep_sf), s, w.ga.row_token, w.ga.flag,
                          w.ga.tok_sf, p->tokens);
    return cuda_check("permute_quant");
  }
  launch_permute_quant(static_cast<const __nv_bfloat16*>(a), a1_gscale, topk_ids, w.seg_base, w.eoff, w.boff,
                       p->tokens, p->hidden, p->experts, p->topk, static_cast<uint8_t*>(rep_fp4), w.lin_sf, c_map, s);
  launch_swizzle_scales(w.lin_sf, w.tile_prefix, w.counts, w.eoff, p->experts, p->hidden,
                        (int64_t)p->tokens * p->topk, static_cast<uint8_t*>(rep_sf), s);
  return cuda_check("permute_quant");
}

int reaxmoe_gemm_w13(const reaxmoe_problem* p, const void* rep_fp4, const void* rep_sf, const void* w1_fp4,
                     const void* w1_sf, const float* w1_alphas, const float* a2_gscale, void* workspace,
                     size_t workspace_bytes, void* int_fp4, void* int_sf, void* stream) {
  int rc = check_problem(p);
  if (rc) return rc;
  Layout L;
  if ((rc = check_ws(p, workspace, workspace_bytes, &L))) return rc;
  if (p->tokens == 0) return 0;
  if (!rep_sf || !w1_fp4 || !w1_sf || !w1_alphas || !a2_gscale || !int_fp4 || !int_sf)
    return fail(REAXMOE_ERR_NULL, "gemm_w13: NULL pointer");
  if (!aligned16(rep_fp4) || !aligned16(rep_sf) || !aligned16(w1_fp4) || !aligned16(w1_sf) || !aligned16(int_fp4))
    return fail(REAXMOE_ERR_MISALIGNED, "gemm_w13: operands must be 16-byte aligned");
  const WS w = carve(workspace, L);
  // rep_fp4 == NULL: the gather layout that reaxmoe_permute_quant left in this workspace
  const GemmLaunch g =
      rep_fp4 != nullptr
          ? w13_launch(p, w, rep_fp4, rep_sf, w1_fp4, w1_sf, w1_alphas, a2_gscale, int_fp4, int_sf)
          : w13_gather_launch(p, w, w.ga.tok_fp4, w.rep_fp4, rep_sf, w1_fp4, w1_sf, w1_alphas, a2_gscale, int_fp4,
                              int_sf);
  if ((rc = launch_grouped_gemm(g, num_sms(), static_cast<cudaStream_t>(stream))))
    return fail(rc, "gemm_w13 launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("gemm_w13");
}

int reaxmoe_gemm_w2(const reaxmoe_problem* p, const void* int_fp4, const void* int_sf, const void* w2_fp4,
                    const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes, void* c3,
                    void* stream) {
  int rc = check_problem(p);
  if (rc) return rc;
  Layout L;
  if ((rc = check_ws(p, workspace, workspace_bytes, &L))) return rc;
  if (p->tokens == 0) return 0;
  if (!int_fp4 || !int_sf || !w2_fp4 || !w2_sf || !w2_alphas || !c3) return fail(REAXMOE_ERR_NULL, "gemm_w2: NULL pointer");
  if (!aligned16(int_fp4) || !aligned16(int_sf) || !aligned16(w2_fp4) || !aligned16(w2_sf) || !aligned16(c3))
    return fail(REAXMOE_ERR_MISALIGNED, "gemm_w2: operands must be 16-byte aligned");
  const WS w = carve(workspace, L);
  const GemmLaunch g = w2_launch(p, w, int_fp4, int_sf, w2_fp4, w2_sf, w2_alphas, c3);
  if ((rc = launch_grouped_gemm(g, num_sms(), static_cast<cudaStream_t>(stream))))
    return fail(rc, "gemm_w2 launch failed: %s", cudaGetErrorString(cudaPeekAtLastError()));
  return cuda_check("gemm_w2");
}

int reaxmoe_combine(const reaxmoe_problem* p, const void* c3, const int32_t* c_map, const float* topk_weights,
                    void* output, void* stream) {
  int rc = check_problem(p);
  if (rc) return rc;
  if (p->tokens == 0) return 0;
  if (!c3 || !c_map || !topk_weights || !output) return fail(REAXMOE_ERR_NULL, "combine: NULL pointer");
  if (!aligned16(c3) || !aligned16(output)) return fail(REAXMOE_ERR_MISALIGNED, "combine: misaligned");
  launch_combine(static_cast<const __nv_bfloat16*>(c3), c_map, topk_weights, p->tokens, p->hidden, p->topk,
                 static_cast<__nv_bfloat16*>(output), num_sms(), static_cast<cudaStream_t>(stream));
  return cuda_check("combine");
}

int reaxmoe_forward(const reaxmoe_forward_args* args, void* workspace, size_t workspace_bytes, void* stream) {
  if (args == nullptr) return fail(REAXMOE_ERR_NULL, "forward: args is NULL");
  const reaxmoe_problem* p = &args->p;
  int rc = check_problem(p);
  if (rc) return rc;
  Layout L;
  if ((rc = check_ws(p, workspace, workspace_bytes, &L))) return rc;
  if (p->tokens == 0) return 0;
  if (!args->a || !args->a1_gscale || !args->w1_fp4 || !args->w1_sf || !args->w1_alphas || !args->a2_gscale ||
      !args->w2_fp4 || !args->w2_sf || !args->w2_alphas || !args->topk_weights || !args->topk_ids || !args->output)
    return fail(REAXMOE_ERR_NULL, "forward: NULL pointer in args");
  if (!aligned16(args->a) || !aligned16(args->w1_fp4) || !aligned16(args->w1_sf) || !aligned16(args->w2_fp4) ||
      !aligned16(args->w2_sf) || !aligned16(args->output))
    return fail(REAXMOE_ERR_MISALIGNED, "forward: activations, weights and output must be 16-byte aligned");
  const WS w = carve(workspace, L);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = do_plan(p, args->topk_ids, w, nullptr, nullptr, s))) return rc;
  // gather layout: token rows quantised once when the experts share their input scale, else per slot
  launch_permute_quant(static_cast<const __nv_bfloat16*>(args->a), args->a1_gscale, args->topk_ids, w.seg_base,
                       w.eoff, w.boff, p->tokens, p->hidden, p->experts, p->topk, w.rep_fp4, w.lin_sf, w.c_map, s,
                       &w.ga);
  launch_swizzle_scales(w.lin_sf, w.tile_prefix, w.counts, w.eoff, p->experts, p->hidden,
                        (int64_t)p->tokens * p->topk, w.rep_sf, s, w.ga.row_token, w.ga.flag, w.ga.tok_sf,
                        p->tokens);
  if ((rc = cuda_check("permute_quant"))) return rc;
  const int sms = num_sms();
  GemmLaunch g1 = w13_gather_launch(p, w, w.ga.tok_fp4, w.rep_fp4, w.rep_sf, args->w1_fp4, args->w1_sf,
                                    args->w1_alphas, args->a2_gscale, w.int_fp4, w.int_sf);
  if ((rc = launch_grouped_gemm(g1, sms, s))) return fail(rc, "forward: gemm_w13 launch failed");
  GemmLaunch g2 = w2_launch(p, w, w.int_fp4, w.int_sf, args->w2_fp4, args->w2_sf, args->w2_alphas, w.c3);
  if ((rc = launch_grouped_gemm(g2, sms, s))) return fail(rc, "forward: gemm_w2 launch failed");
  launch_combine(w.c3, w.c_map, args->topk_weights, p->tokens, p->hidden, p->topk,
                 static_cast<__nv_bfloat16*>(args->output), sms, s);
  return cuda_check("forward");
}

int reaxmoe_forward_prequant(const reaxmoe_forward_args* args, const void* a_scales, float a_gscale,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (args == nullptr) return fail(REAXMOE_ERR_NULL, "forward_prequant: args is NULL");
  const reaxmoe_problem* p = &args->p;
  int rc = check_problem(p);
  if (rc) return rc;
  if (p->hidden > 4096 || p->hidden % 256 != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "forward_prequant: hidden=%d (a multiple of 256, <= 4096)", p->hidden);
  if (!(a_gscale > 0.0f)) return fail(REAXMOE_ERR_BAD_SHAPE, "forward_prequant: a_gscale must be > 0");
  Layout L;
  if ((rc = check_ws(p, workspace, workspace_bytes, &L))) return rc;
  if (p->tokens == 0) return 0;
  if (!args->a || !a_scales || !args->a1_gscale || !args->w1_fp4 || !args->w1_sf || !args->w1_alphas ||
      !args->a2_gscale || !args->w2_fp4 || !args->w2_sf || !args->w2_alphas || !args->topk_weights ||
      !args->topk_ids || !args->output)
    return fail(REAXMOE_ERR_NULL, "forward_prequant: NULL pointer in args");
  if (!aligned16(args->a) || !aligned16(a_scales) || !aligned16(args->w1_fp4) || !aligned16(args->w1_sf) ||
      !aligned16(args->w2_fp4) || !aligned16(args->w2_sf) || !aligned16(args->output))
    return fail(REAXMOE_ERR_MISALIGNED, "forward_prequant: activations, weights and output must be 16-byte aligned");
  const WS w = carve(workspace, L);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = do_plan(p, args->topk_ids, w, nullptr, nullptr, s))) return rc;
  // gather layout: the GEMM and the scale swizzle read the caller's token rows in place through the slot map
  launch_permute_fp4(static_cast<const uint8_t*>(args->a), static_cast<const uint8_t*>(a_scales), a_gscale,
                     args->a1_gscale, args->topk_ids, w.seg_base, w.eoff, p->tokens, p->hidden, p->experts, p->topk,
                     w.rep_fp4, w.lin_sf, w.c_map, w.status, s, &w.ga);
  launch_swizzle_scales(w.lin_sf, w.tile_prefix, w.counts, w.eoff, p->experts, p->hidden,
                        (int64_t)p->tokens * p->topk, w.rep_sf, s, w.ga.row_token, w.ga.flag,
                        static_cast<const uint8_t*>(a_scales), p->tokens);
  if ((rc = cuda_check("permute_fp4"))) return rc;
  const int sms = num_sms();
  GemmLaunch g1 = w13_gather_launch(p, w, args->a, w.rep_fp4, w.rep_sf, args->w1_fp4, args->w1_sf, args->w1_alphas,
                                    args->a2_gscale, w.int_fp4, w.int_sf);
  if ((rc = launch_grouped_gemm(g1, sms, s))) return fail(rc, "forward_prequant: gemm_w13 launch failed");
  GemmLaunch g2 = w2_launch(p, w, w.int_fp4, w.int_sf, args->w2_fp4, args->w2_sf, args->w2_alphas, w.c3);
  if ((rc = launch_grouped_gemm(g2, sms, s))) return fail(rc, "forward_prequant: gemm_w2 launch failed");
  launch_combine(w.c3, w.c_map, args->topk_weights, p->tokens, p->hidden, p->topk,
                 static_cast<__nv_bfloat16*>(args->output), sms, s);
  return cuda_check("forward_prequant");
}

int reaxmoe_quantize(const void* x, int32_t x_is_fp32, int64_t rows, int32_t cols, int32_t group_rows,
                     const float* gscale, void* packed, void* scales, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 64 != 0 || group_rows <= 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "quantize: rows=%lld cols=%d group_rows=%d", (long long)rows, cols, group_rows);
  if (rows == 0) return 0;
  if (!x || !gscale || !packed || !scales) return fail(REAXMOE_ERR_NULL, "quantize: NULL pointer");
  if (!aligned16(x) || !aligned16(packed) || !aligned16(scales))
    return fail(REAXMOE_ERR_MISALIGNED, "quantize: pointers must be 16-byte aligned");
  launch_quantize(x, x_is_fp32 != 0, rows, cols, group_rows, gscale, static_cast<uint8_t*>(packed),
                  static_cast<uint8_t*>(scales), static_cast<cudaStream_t>(stream));
  return cuda_check("quantize");
}

int reaxmoe_prepack_w13(const void* w1_fp4, const void* w1_sf, int32_t experts, int32_t inter, int32_t hidden,
                        void* w1p_fp4, void* w1p_sf, void* stream) {
  if (experts < 1 || inter < 64 || inter % 64 != 0 || hidden < 128 || hidden % 128 != 0)
    return fail(REAXMOE_ERR_BAD_SHAPE, "prepack_w13: experts=%d inter=%d hidden=%d", experts, inter, hidden);
  if (!w1_fp4 || !w1_sf || !w1p_fp4 || !w1p_sf) return fail(REAXMOE_ERR_NULL, "prepack_w13: NULL pointer");
  if (w1_fp4 == w1p_fp4 || w1_sf == w1p_sf) return fail(REAXMOE_ERR_BAD_SHAPE, "prepack_w13: in-place not allowed");
  if (!aligned16(w1_fp4) || !aligned16(w1p_fp4)) return fail(REAXMOE_ERR_MISALIGNED, "prepack_w13: misaligned");
  launch_prepack_w13(static_cast<const uint8_t*>(w1_fp4), static_cast<const uint8_t*>(w1_sf), experts, inter, hidden,
                     static_cast<uint8_t*>(w1p_fp4), static_cast<uint8_t*>(w1p_sf), static_cast<cudaStream_t>(stream));
  return cuda_check("prepack_w13");
}

size_t reaxmoe_ep_record_bytes(int32_t hidden, int32_t topk) {
  if (hidden < 128 || hidden % 128 != 0 || topk < 1 || topk > kMaxTopk) return 0;
  const size_t b = (size_t)hidden / 2 + (size_t)hidden / 16 + (size_t)topk * 8;
  return (b + 15) & ~size_t(15);
}

size_t reaxmoe_ep_dispatch_workspace_size(const reaxmoe_problem* p, int32_t ranks) {
  if (check_ep(p, ranks)) return 0;
  return ep_dispatch_layout(p, ranks).total;
}

// The dispatch's routing steps (rank ids, counts, plan) into the workspace; send_counts [ranks] on the device.
static int ep_dispatch_plan(const reaxmoe_problem* p, int ranks, const float* a1_gscale, const int32_t* topk_ids,
                            void* workspace, size_t workspace_bytes, int32_t* send_counts, cudaStream_t s,
                            const char* who) {
  int rc = check_ep(p, ranks);
  if (rc) return rc;
  const EpDispatchLayout L = ep_dispatch_layout(p, ranks);
  if (workspace == nullptr) return fail(REAXMOE_ERR_WORKSPACE, "%s: workspace is NULL", who);
  if (!aligned16(workspace)) return fail(REAXMOE_ERR_MISALIGNED, "%s: workspace not 16-byte aligned", who);
  if (workspace_bytes < L.total)
    return fail(REAXMOE_ERR_WORKSPACE, "%s: workspace %zu bytes < required %zu", who, workspace_bytes, L.total);
  if (send_counts == nullptr) return fail(REAXMOE_ERR_NULL, "%s: send_counts is NULL", who);
  uint8_t* b = static_cast<uint8_t*>(workspace);
  cudaMemsetAsync(b + L.status, 0, sizeof(int), s);
  if (p->tokens == 0) {
    cudaMemsetAsync(send_counts, 0, (size_t)ranks * 4, s);
    return 0;
  }
  if (!a1_gscale || !topk_ids) return fail(REAXMOE_ERR_NULL, "%s: NULL pointer", who);
  const int El = p->experts / ranks;
  int* rid = reinterpret_cast<int*>(b + L.rid);
  int* seg_counts = reinterpret_cast<int*>(b + L.seg_counts);
  launch_ep_rank_ids(topk_ids, p->tokens, p->topk, p->experts, El, a1_gscale, rid,
                     reinterpret_cast<int*>(b + L.status), s);
  launch_count(rid, p->tokens, p->topk, ranks, seg_counts, reinterpret_cast<int*>(b + L.status), s);
  launch_plan(seg_counts, (int)ceil_div64(p->tokens, kSegTokens), ranks, reinterpret_cast<int*>(b + L.seg_base),
              send_counts, reinterpret_cast<int*>(b + L.roff), reinterpret_cast<int*>(b + L.boff),
              reinterpret_cast<int*>(b + L.tile_prefix), nullptr, nullptr, 0, 0, 0, 0, s);
  return 0;
}

int reaxmoe_ep_dispatch(const reaxmoe_problem* p, int32_t ranks, const void* a, const float* a1_gscale,
                        const int32_t* topk_ids, const float* topk_weights, void* workspace, size_t workspace_bytes,
                        int32_t* send_counts, int32_t* send_map, void* send_records, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = ep_dispatch_plan(p, ranks, a1_gscale, topk_ids, workspace, workspace_bytes, send_counts, s,
                            "ep_dispatch");
  if (rc) return rc;
  if (p->tokens == 0) return cuda_check("ep_dispatch");
  if (!a || !topk_weights || !send_map || !send_records) return fail(REAXMOE_ERR_NULL, "ep_dispatch: NULL pointer");
  if (!aligned16(a) || !aligned16(send_records))
    return fail(REAXMOE_ERR_MISALIGNED, "ep_dispatch: a and send_records must be 16-byte aligned");
  const EpDispatchLayout L = ep_dispatch_layout(p, ranks);
  const int El = p->experts / ranks;
  const int rec = (int)reaxmoe_ep_record_bytes(p->hidden, p->topk);
  uint8_t* b = static_cast<uint8_t*>(workspace);
  launch_ep_pack(static_cast<const __nv_bfloat16*>(a), a1_gscale, topk_ids, topk_weights,
                 reinterpret_cast<const int*>(b + L.rid), reinterpret_cast<const int*>(b + L.seg_base),
                 reinterpret_cast<const int*>(b + L.roff), p->tokens, p->hidden, p->experts, El, p->topk, rec,
                 static_cast<uint8_t*>(send_records), send_map, s);
  return cuda_check("ep_dispatch");
}

int reaxmoe_ep_dispatch_plan(const reaxmoe_problem* p, int32_t ranks, const float* a1_gscale,
                             const int32_t* topk_ids, void* workspace, size_t workspace_bytes, int32_t* send_counts,
                             void* stream) {
  int rc = ep_dispatch_plan(p, ranks, a1_gscale, topk_ids, workspace, workspace_bytes, send_counts,
                            static_cast<cudaStream_t>(stream), "ep_dispatch_plan");
  return rc ? rc : cuda_check("ep_dispatch_plan");
}

int reaxmoe_ep_dispatch_pack(const reaxmoe_problem* p, int32_t ranks, const void* a, const float* a1_gscale,
                             const int32_t* topk_ids, const float* topk_weights, const void* workspace,
                             size_t workspace_bytes, int32_t* send_map, const uint64_t* records, void* stream) {
  int rc = check_ep(p, ranks);
  if (rc) return rc;
  const EpDispatchLayout L = ep_dispatch_layout(p, ranks);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(REAXMOE_ERR_WORKSPACE, "ep_dispatch_pack: workspace missing or smaller than %zu bytes", L.total);
  if (p->tokens == 0) return 0;
  if (!a || !a1_gscale || !topk_ids || !topk_weights || !send_map || !records)
    return fail(REAXMOE_ERR_NULL, "ep_dispatch_pack: NULL pointer");
  const int rec = (int)reaxmoe_ep_record_bytes(p->hidden, p->topk);
  PeerPtrs dst{};
  for (int d = 0; d < ranks; ++d) {
    if (records[d] == 0 || records[d] % 16 != 0)
      return fail(REAXMOE_ERR_MISALIGNED, "ep_dispatch_pack: records[%d] is NULL or not 16-byte aligned", d);
    dst.p[d] = records[d];
  }
  if (!aligned16(a)) return fail(REAXMOE_ERR_MISALIGNED, "ep_dispatch_pack: a must be 16-byte aligned");
  const uint8_t* b = static_cast<const uint8_t*>(workspace);
  launch_ep_pack_peer(static_cast<const __nv_bfloat16*>(a), a1_gscale, topk_ids, topk_weights,
                      reinterpret_cast<const int*>(b + L.rid), reinterpret_cast<const int*>(b + L.seg_base),
                      reinterpret_cast<const int*>(b + L.roff), p->tokens, p->hidden, p->experts,
                      p->experts / ranks, p->topk, rec, dst, send_map, static_cast<cudaStream_t>(stream));
  return cuda_check("ep_dispatch_pack");
}

size_t reaxmoe_ep_expert_workspace_size(const reaxmoe_problem* local) {
  if (check_problem(local, true)) return 0;
  return ep_expert_total(local, layout(local));
}

// The receiver's steps; the pre-summed rows go to `partial` (route == nullptr) or along `route`.
static int ep_expert_forward(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                             const void* w1_sf, const float* w1_alphas, const float* a2_gscale, const void* w2_fp4,
                             const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes,
                             void* partial, const RowRoute* route, cudaStream_t s, const char* who) {
  const reaxmoe_problem* p = local;
  int rc = check_problem(p, true);
  if (rc) return rc;
  const Layout L = layout(p);
  const size_t need = ep_expert_total(p, L);
  if (workspace == nullptr) return fail(REAXMOE_ERR_WORKSPACE, "%s: workspace is NULL", who);
  if (!aligned16(workspace)) return fail(REAXMOE_ERR_MISALIGNED, "%s: workspace not 16-byte aligned", who);
  if (workspace_bytes < need)
    return fail(REAXMOE_ERR_WORKSPACE, "%s: workspace %zu bytes < required %zu", who, workspace_bytes, need);
  if (p->tokens == 0) return 0;
  if (!recv_records || !w1_fp4 || !w1_sf || !w1_alphas || !a2_gscale || !w2_fp4 || !w2_sf || !w2_alphas ||
      (!partial && !route))
    return fail(REAXMOE_ERR_NULL, "%s: NULL pointer", who);
  if (!aligned16(recv_records) || !aligned16(w1_fp4) || !aligned16(w1_sf) || !aligned16(w2_fp4) ||
      !aligned16(w2_sf) || (partial && !aligned16(partial)))
    return fail(REAXMOE_ERR_MISALIGNED, "%s: records, weights and partial must be 16-byte aligned", who);
  const WS w = carve(workspace, L);
  uint8_t* b = static_cast<uint8_t*>(workspace);
  int* lid = reinterpret_cast<int*>(b + ep_expert_lid(L));
  float* lw = reinterpret_cast<float*>(b + ep_expert_lw(p, L));
  const uint8_t* rec = static_cast<const uint8_t*>(recv_records);
  const int rec_bytes = (int)reaxmoe_ep_record_bytes(p->hidden, p->topk);
  launch_ep_unpack_meta(rec, p->tokens, p->topk, p->hidden, rec_bytes, lid, lw, s);
  if ((rc = do_plan(p, lid, w, nullptr, nullptr, s))) return rc;
  // gather layout: w13 and the scale swizzle read each slot's FP4 row and scale row inside its record
  launch_ep_permute(rec, lid, w.seg_base, w.eoff, p->tokens, p->hidden, p->experts, p->topk, rec_bytes, w.rep_fp4,
                    w.lin_sf, w.c_map, s, &w.ga);
  launch_swizzle_scales(w.lin_sf, w.tile_prefix, w.counts, w.eoff, p->experts, p->hidden,
                        (int64_t)p->tokens * p->topk, w.rep_sf, s, w.ga.row_token, w.ga.flag, rec + p->hidden / 2,
                        p->tokens, rec_bytes);
  if ((rc = cuda_check("ep_permute"))) return rc;
  const int sms = num_sms();
  GemmLaunch g1 = w13_gather_launch(p, w, rec, w.rep_fp4, w.rep_sf, w1_fp4, w1_sf, w1_alphas, a2_gscale, w.int_fp4,
                                    w.int_sf);
  g1.tok_stride = rec_bytes;
  if ((rc = launch_grouped_gemm(g1, sms, s))) return fail(rc, "%s: gemm_w13 launch failed", who);
  GemmLaunch g2 = w2_launch(p, w, w.int_fp4, w.int_sf, w2_fp4, w2_sf, w2_alphas, w.c3);
  if (route != nullptr && route->skip_single) {
    // records with one local pair: the w2 epilogue stores their finished rows straight to the source rank
    uint64_t* direct_dst = reinterpret_cast<uint64_t*>(b + ep_expert_direct(p, L));
    float* direct_w = reinterpret_cast<float*>(b + ep_expert_direct_w(p, L));
    launch_ep_direct(w.c_map, lw, p->tokens, p->topk, p->hidden, *route, direct_dst, direct_w, s);
    g2.direct_dst = direct_dst;
    g2.direct_w = direct_w;
    g2.topk = p->topk;
  }
  if ((rc = launch_grouped_gemm(g2, sms, s))) return fail(rc, "%s: gemm_w2 launch failed", who);
  if (route != nullptr)
    launch_combine_routed(w.c3, w.c_map, lw, p->tokens, p->hidden, p->topk, *route, sms, s);
  else
    launch_combine(w.c3, w.c_map, lw, p->tokens, p->hidden, p->topk, static_cast<__nv_bfloat16*>(partial), sms, s);
  return cuda_check(who);
}

int reaxmoe_ep_expert_forward(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                              const void* w1_sf, const float* w1_alphas, const float* a2_gscale, const void* w2_fp4,
                              const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes,
                              void* partial, void* stream) {
  return ep_expert_forward(local, recv_records, w1_fp4, w1_sf, w1_alphas, a2_gscale, w2_fp4, w2_sf, w2_alphas,
                           workspace, workspace_bytes, partial, nullptr, static_cast<cudaStream_t>(stream),
                           "ep_expert_forward");
}

int reaxmoe_ep_expert_forward_to(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                                 const void* w1_sf, const float* w1_alphas, const float* a2_gscale,
                                 const void* w2_fp4, const void* w2_sf, const float* w2_alphas, void* workspace,
                                 size_t workspace_bytes, int32_t ranks, const int64_t* bounds, const uint64_t* rows,
                                 void* stream) {
  if (ranks < 1 || ranks > kMaxRanks) return fail(REAXMOE_ERR_BAD_SHAPE, "ep_expert_forward_to: ranks=%d", ranks);
  if (local == nullptr || bounds == nullptr || rows == nullptr)
    return fail(REAXMOE_ERR_NULL, "ep_expert_forward_to: NULL pointer");
  if (bounds[0] != 0 || bounds[ranks] != local->tokens)
    return fail(REAXMOE_ERR_BAD_SHAPE, "ep_expert_forward_to: bounds must run from 0 to tokens=%d", local->tokens);
  RowRoute route{};
  route.ranks = ranks;
  route.skip_single = ep_direct_rows() ? 1 : 0;
  for (int q = 0; q <= ranks; ++q) {
    if (q > 0 && bounds[q] < bounds[q - 1])
      return fail(REAXMOE_ERR_BAD_SHAPE, "ep_expert_forward_to: bounds decrease at %d", q);
    route.bound[q] = bounds[q];
  }
  for (int q = 0; q < ranks; ++q) {
    if (bounds[q + 1] > bounds[q] && (rows[q] == 0 || rows[q] % 32 != 0))
      return fail(REAXMOE_ERR_MISALIGNED, "ep_expert_forward_to: rows[%d] is NULL or not 32-byte aligned", q);
    route.p[q] = rows[q];
  }
  return ep_expert_forward(local, recv_records, w1_fp4, w1_sf, w1_alphas, a2_gscale, w2_fp4, w2_sf, w2_alphas,
                           workspace, workspace_bytes, nullptr, &route, static_cast<cudaStream_t>(stream),
                           "ep_expert_forward_to");
}

// ---- the receiver in two calls, so that the row stores of one part of the received records run beside the GEMMs of
// the next part (on another stream, pinned to a few SMs)
int reaxmoe_ep_expert_gemms(const reaxmoe_problem* local, const void* recv_records, const void* w1_fp4,
                            const void* w1_sf, const float* w1_alphas, const float* a2_gscale, const void* w2_fp4,
                            const void* w2_sf, const float* w2_alphas, void* workspace, size_t workspace_bytes,
                            int32_t sm_limit, void* stream) {
  const reaxmoe_problem* p = local;
  int rc = check_problem(p, true);
  if (rc) return rc;
  const Layout L = layout(p);
  const size_t need = ep_expert_total(p, L);
  if (workspace == nullptr) return fail(REAXMOE_ERR_WORKSPACE, "ep_expert_gemms: workspace is NULL");
  if (!aligned16(workspace)) return fail(REAXMOE_ERR_MISALIGNED, "ep_expert_gemms: workspace not 16-byte aligned");
  if (workspace_bytes < need)
    return fail(REAXMOE_ERR_WORKSPACE, "ep_expert_gemms: workspace %zu bytes < required %zu", workspace_bytes, need);
  if (sm_limit < 0) return fail(REAXMOE_ERR_BAD_SHAPE, "ep_expert_gemms: sm_limit=%d", sm_limit);
  if (p->tokens == 0) return 0;
  if (!recv_records || !w1_fp4 || !w1_sf || !w1_alphas || !a2_gscale || !w2_fp4 || !w2_sf || !w2_alphas)
    return fail(REAXMOE_ERR_NULL, "ep_expert_gemms: NULL pointer");
  if (!aligned16(recv_records) || !aligned16(w1_fp4) || !aligned16(w1_sf) || !aligned16(w2_fp4) || !aligned16(w2_sf))
    return fail(REAXMOE_ERR_MISALIGNED, "ep_expert_gemms: records and weights must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const WS w = carve(workspace, L);
  uint8_t* b = static_cast<uint8_t*>(workspace);
  int* lid = reinterpret_cast<int*>(b + ep_expert_lid(L));
  float* lw = reinterpret_cast<float*>(b + ep_expert_lw(p, L));
  const uint8_t* rec = static_cast<const uint8_t*>(recv_records);
  const int rec_bytes = (int)reaxmoe_ep_record_bytes(p->hidden, p->topk);
  launch_ep_unpack_meta(rec, p->tokens, p->topk, p->hidden, rec_bytes, lid, lw, s);
  if ((rc = do_plan(p, lid, w, nullptr, nullptr, s))) return rc;
  // gather layout: w13 and the scale swizzle read each slot's FP4 row and scale row inside its record
  launch_ep_permute(rec, lid, w.seg_base, w.eoff, p->tokens, p->hidden, p->experts, p->topk, rec_bytes, w.rep_fp4,
                    w.lin_sf, w.c_map, s, &w.ga);
  launch_swizzle_scales(w.lin_sf, w.tile_prefix, w.counts, w.eoff, p->experts, p->hidden,
                        (int64_t)p->tokens * p->topk, w.rep_sf, s, w.ga.row_token, w.ga.flag, rec + p->hidden / 2,
                        p->tokens, rec_bytes);
  if ((rc = cuda_check("ep_expert_gemms permute"))) return rc;
  const int sms = sm_limit > 0 && sm_limit < num_sms() ? sm_limit : num_sms();
  GemmLaunch g1 = w13_gather_launch(p, w, rec, w.rep_fp4, w.rep_sf, w1_fp4, w1_sf, w1_alphas, a2_gscale, w.int_fp4,
                                    w.int_sf);
  g1.tok_stride = rec_bytes;
  if ((rc = launch_grouped_gemm(g1, sms, s))) return fail(rc, "ep_expert_gemms: gemm_w13 launch failed");
  GemmLaunch g2 = w2_launch(p, w, w.int_fp4, w.int_sf, w2_fp4, w2_sf, w2_alphas, w.c3);
  if ((rc = launch_grouped_gemm(g2, sms, s))) return fail(rc, "ep_expert_gemms: gemm_w2 launch failed");
  return cuda_check("ep_expert_gemms");
}

int reaxmoe_ep_presum_to(const reaxmoe_problem* local, const void* workspace, size_t workspace_bytes, int32_t ranks,
                         const int64_t* bounds, const uint64_t* rows, int32_t sms, void* stream) {
  int rc = check_problem(local, true);
  if (rc) return rc;
  const Layout L = layout(local);
  if (workspace == nullptr || workspace_bytes < ep_expert_total(local, L))
    return fail(REAXMOE_ERR_WORKSPACE, "ep_presum_to: workspace missing or smaller than the gemms call's");
  if (ranks < 1 || ranks > kMaxRanks) return fail(REAXMOE_ERR_BAD_SHAPE, "ep_presum_to: ranks=%d", ranks);
  if (bounds == nullptr || rows == nullptr) return fail(REAXMOE_ERR_NULL, "ep_presum_to: NULL pointer");
  if (bounds[0] != 0 || bounds[ranks] != local->tokens)
    return fail(REAXMOE_ERR_BAD_SHAPE, "ep_presum_to: bounds must run from 0 to tokens=%d", local->tokens);
  if (sms < 0) return fail(REAXMOE_ERR_BAD_SHAPE, "ep_presum_to: sms=%d", sms);
  RowRoute route{};
  route.ranks = ranks;
  route.skip_single = 0;
  for (int q = 0; q <= ranks; ++q) {
    if (q > 0 && bounds[q] < bounds[q - 1])
      return fail(REAXMOE_ERR_BAD_SHAPE, "ep_presum_to: bounds decrease at %d", q);
    route.bound[q] = bounds[q];
  }
  for (int q = 0; q < ranks; ++q) {
    if (bounds[q + 1] > bounds[q] && (rows[q] == 0 || rows[q] % 32 != 0))
      return fail(REAXMOE_ERR_MISALIGNED, "ep_presum_to: rows[%d] is NULL or not 32-byte aligned", q);
    route.p[q] = rows[q];
  }
  if (local->tokens == 0) return 0;
  const WS w = carve(const_cast<void*>(workspace), L);
  const float* lw = reinterpret_cast<const float*>(static_cast<const uint8_t*>(workspace) + ep_expert_lw(local, L));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (sms > 0)
    rc = launch_combine_routed_pinned(w.c3, w.c_map, lw, local->tokens, local->hidden, local->topk, route,
                                      sms < num_sms() ? sms : num_sms(), s);
  else
    rc = launch_combine_routed(w.c3, w.c_map, lw, local->tokens, local->hidden, local->topk, route, num_sms(), s);
  if (rc) return fail(REAXMOE_ERR_CUDA, "ep_presum_to: launch failed");
  return cuda_check("ep_presum_to");
}

int reaxmoe_ep_copy_rows(int32_t n, const uint64_t* dst, const uint64_t* src, const uint64_t* bytes, void* stream) {
  if (n < 0) return fail(REAXMOE_ERR_BAD_SHAPE, "ep_copy_rows: n=%d", n);
  if (n > 0 && (dst == nullptr || src == nullptr || bytes == nullptr))
    return fail(REAXMOE_ERR_NULL, "ep_copy_rows: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    if (bytes[i] == 0) continue;
    if (dst[i] == 0 || src[i] == 0) return fail(REAXMOE_ERR_NULL, "ep_copy_rows: copy %d has a NULL address", i);
    // one plain copy per range: the copy engines move it (over NVLink when dst is a peer's mapped buffer)
    if (cudaMemcpyAsync(reinterpret_cast<void*>(dst[i]), reinterpret_cast<const void*>(src[i]), (size_t)bytes[i],
                        cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return fail(REAXMOE_ERR_CUDA, "ep_copy_rows: copy %d failed", i);
  }
  return 0;
}

int reaxmoe_ep_combine(int32_t tokens, int32_t hidden, int32_t topk, const int32_t* send_map, const void* returned,
                       void* output, void* stream) {
  if (tokens < 0 || hidden < 128 || hidden % 128 != 0 || topk < 1 || topk > kMaxTopk)
    return fail(REAXMOE_ERR_BAD_SHAPE, "ep_combine: tokens=%d hidden=%d topk=%d", tokens, hidden, topk);
  if (tokens == 0) return 0;
  if (!send_map || !returned || !output) return fail(REAXMOE_ERR_NULL, "ep_combine: NULL pointer");
  if (!aligned16(returned) || !aligned16(output)) return fail(REAXMOE_ERR_MISALIGNED, "ep_combine: misaligned");
  launch_ep_combine(static_cast<const __nv_bfloat16*>(returned), send_map, tokens, hidden, topk,
                    static_cast<__nv_bfloat16*>(output), num_sms(), static_cast<cudaStream_t>(stream));
  return cuda_check("ep_combine");
}

size_t reaxmoe_ep_signal_bytes(void) { return up256(kSigBytes); }

int reaxmoe_ep_signal(int32_t ranks, int32_t rank, const uint64_t* blocks, uint32_t epoch,
                      const int32_t* send_counts, uint64_t timeout_ns, void* stream) {
  if (ranks < 1 || ranks > kMaxRanks || rank < 0 || rank >= ranks)
    return fail(REAXMOE_ERR_BAD_SHAPE, "ep_signal: rank=%d ranks=%d", rank, ranks);
  if (blocks == nullptr) return fail(REAXMOE_ERR_NULL, "ep_signal: blocks is NULL");
  PeerPtrs b{};
  for (int d = 0; d < ranks; ++d) {
    if (blocks[d] == 0 || blocks[d] % 256 != 0)
      return fail(REAXMOE_ERR_MISALIGNED, "ep_signal: blocks[%d] is NULL or not 256-byte aligned", d);
    b.p[d] = blocks[d];
  }
  launch_ep_signal(b, rank, ranks, epoch, send_counts, (unsigned long long)timeout_ns,
                   static_cast<cudaStream_t>(stream));
  return cuda_check("ep_signal");
}

int reaxmoe_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return fail(REAXMOE_ERR_NULL, "ipc_alloc: bad argument");
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess)
    return fail(REAXMOE_ERR_CUDA, "ipc_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(cudaGetLastError()));
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    cudaFree(p);
    return fail(REAXMOE_ERR_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return 0;
}

int reaxmoe_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(REAXMOE_ERR_NULL, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return fail(REAXMOE_ERR_CUDA, "ipc_open: %s", cudaGetErrorString(cudaGetLastError()));
  return 0;
}

int reaxmoe_ipc_close(void* ptr) {
  if (ptr != nullptr && cudaIpcCloseMemHandle(ptr) != cudaSuccess)
    return fail(REAXMOE_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(cudaGetLastError()));
  return 0;
}

int reaxmoe_ipc_free(void* ptr) {
  if (ptr != nullptr && cudaFree(ptr) != cudaSuccess)
    return fail(REAXMOE_ERR_CUDA, "ipc_free: %s", cudaGetErrorString(cudaGetLastError()));
  return 0;
}

int reaxmoe_read_status(void* workspace, size_t workspace_bytes, int32_t clear, void* stream) {
  if (workspace == nullptr || workspace_bytes < 64) return fail(REAXMOE_ERR_WORKSPACE, "read_status: bad workspace");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return fail(REAXMOE_ERR_CUDA, "read_status: %s", cudaGetErrorString(cudaGetLastError()));
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyAsync(workspace, &zero, sizeof(int), cudaMemcpyHostToDevice, s);
    cudaStreamSynchronize(s);
  }
  return v;
}

}  // extern "C"
