// C-ABI entry points that compose the kernels: expert projections (GEMV or
// tcgen05 grouped GEMM), mxfp4_matmul, and the whole-layer forward.
#include <nvtx3/nvToolsExt.h>

#include "bs_common.cuh"

namespace bs {

// NVTX range over one stage's launches (host-side; nsys/ncu show it beside
// the kernels; costs nothing without a profiler attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
};

int router_launch(const void* x, int x_dtype, const void* weight, const void* bias, int w_dtype,
                  int64_t T, int64_t H, int64_t E, int64_t k, float* logits, float* scores,
                  void* indices, int index_dtype, void* ws, size_t ws_bytes, cudaStream_t st);
size_t router_workspace_bytes(int64_t T, int64_t H, int64_t E, int w_dtype);
size_t dispatch_workspace_bytes(int64_t T, int64_t k, int64_t E);
int dispatch_launch(const void* indices, int index_dtype, int64_t T, int64_t k, int64_t E,
                    const void* x, int64_t H, int32_t* offsets, int32_t* row_of_slot,
                    int32_t* token_of_row, void* x_perm, void* ws, size_t ws_bytes,
                    cudaStream_t st);
int rmsnorm_launch(const void* x, int64_t T, int64_t H, const void* weight, int w_dtype, float eps, void* out,
                   cudaStream_t st);
int combine_launch(const void* y, const int32_t* row_of_slot, const float* weights, int64_t T,
                   int64_t k, int64_t H, void* out, cudaStream_t st,
                   const void* residual = nullptr);
int gemv_gate_up_launch(const void* x, const int32_t* offsets, int64_t rows_total, int64_t E,
                        int64_t H, int64_t I, const void* blocks, const void* scales,
                        const void* bias, int bias_f32, float alpha, float limit, void* h,
                        cudaStream_t st);
int gemv_plain_launch(const void* x, const int32_t* offsets, int64_t rows_total, int64_t E,
                      int64_t K, int64_t N, const void* blocks, const void* scales,
                      const void* bias, int bias_f32, void* y, cudaStream_t st);
// tcgen05 grouped GEMM (grouped_gemm.cu).  mode 0: gate_up + SwiGLU, 1: plain + bias.
int tc_grouped_launch(int mode, const void* x, const int32_t* offsets, int64_t rows_total,
                      int64_t max_rows_per_expert, int64_t E, int64_t K, int64_t N,
                      const void* blocks, const void* scales, const void* bias, int bias_f32,
                      float alpha, float limit, void* out, cudaStream_t st);
bool tc_supported(const void* scales, int64_t K, int64_t N);
int tc_pair_launch(int mode, const void* x, const int32_t* offsets, int64_t rows_total,
                   int64_t max_rows_per_expert, int64_t E, int64_t K, int64_t N, const void* blocks,
                   const void* scales, const void* bias, int bias_f32, float alpha, float limit, void* out,
                   cudaStream_t st);
// Decode path (decode.cu): router + dispatch + block-scaled expert MMAs + combine, T <= 64.
bool decode_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k);
size_t decode_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k);
int decode_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                   const void* rw, const void* rb, int rdt, float* scores, int32_t* indices,
                   const void* gu_b, const void* gu_s, const void* gu_bias, const void* dn_b,
                   const void* dn_s, const void* dn_bias, int bias_f32, float alpha, float limit,
                   void* out, void* ws, cudaStream_t st,
                   const void* residual = nullptr);
// Fused decode kernel (decode_fused.cu): the whole layer in one cooperative launch, T <= 8.
bool fused_supported(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, float alpha, float limit,
                     const void* gu_b, const void* gu_s, const void* dn_b, const void* dn_s);
size_t fused_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k);
int fused_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k, const void* rw,
                  const void* rb, int rdt, float* scores, int32_t* indices, const void* gu_b, const void* gu_s,
                  const void* gu_bias, const void* dn_b, const void* dn_s, const void* dn_bias, int bias_f32,
                  float alpha, float limit, void* out, void* ws, cudaStream_t st, const void* residual);

namespace {

// Tokens per expert above which the tensor-core path wins over the GEMV.
constexpr int64_t kGemvMaxRowsPerExpert = 16;

// AUTO: the GEMV at few tokens per expert; the tensor-core kernel otherwise,
// when the scale rows can be bulk-copied (16-byte aligned runs).
int pick_algo(int algo, int64_t rows_total, int64_t E, const void* scales, int64_t K, int64_t N) {
  if (algo != BS_ALGO_AUTO) return algo;
  if (rows_total <= kGemvMaxRowsPerExpert * E) return BS_ALGO_GEMV;
  return tc_supported(scales, K, N) ? BS_ALGO_TCGEN05 : BS_ALGO_GEMV;
}

int check_expert_args(const char* fn, const void* x, const void* blocks, const void* scales,
                      const void* out, int64_t rows_total, int64_t E, int64_t K, int64_t N,
                      int bias_dtype, int algo) {
  BS_ARG(x && blocks && scales && out, "%s: null pointer", fn);
  BS_ARG(rows_total >= 0 && E > 0 && K > 0 && N > 0, "%s: bad sizes", fn);
  BS_ARG(K % 32 == 0, "%s: contraction size %lld is not a multiple of 32", fn, (long long)K);
  BS_ARG(E <= 1024, "%s: at most 1024 experts", fn);
  BS_ARG(rows_total < (int64_t)INT32_MAX && N < (int64_t)INT32_MAX, "%s: sizes too large", fn);
  BS_ARG(bias_dtype == BS_BF16 || bias_dtype == BS_F32, "%s: bias dtype must be bf16 or f32", fn);
  BS_ARG((algo >= BS_ALGO_AUTO && algo <= BS_ALGO_TCGEN05) || algo == BS_ALGO_TCGEN05_PAIR,
         "%s: unknown algo %d", fn, algo);
  BS_ALIGNED16(x, "x");
  BS_ALIGNED16(blocks, "blocks");
  return BS_OK;
}

}  // namespace

int gate_up(const void* x, const int32_t* offsets, int64_t rows_total, int64_t max_rows, int64_t E,
            int64_t H, int64_t I, const void* blocks, const void* scales, const void* bias,
            int bias_dtype, float alpha, float limit, void* h, int algo, cudaStream_t st) {
  BS_TRY(check_expert_args("bs_moe_gate_up", x, blocks, scales, h, rows_total, E, H, 2 * I,
                           bias_dtype, algo));
  BS_ARG(offsets, "bs_moe_gate_up: null expert_offsets");
  BS_ARG(I % 8 == 0, "bs_moe_gate_up: intermediate size must be a multiple of 8");
  if (rows_total == 0) return BS_OK;
  BS_TRY(check_device());
  const int a = pick_algo(algo, rows_total, E, scales, H, 2 * I);
  const int bf32 = bias_dtype == BS_F32;
  if (a == BS_ALGO_GEMV)
    return gemv_gate_up_launch(x, offsets, rows_total, E, H, I, blocks, scales, bias, bf32, alpha,
                               limit, h, st);
  auto launch = a == BS_ALGO_TCGEN05_PAIR ? tc_pair_launch : tc_grouped_launch;
  return launch(0, x, offsets, rows_total, max_rows, E, H, 2 * I, blocks, scales, bias, bf32, alpha, limit, h, st);
}

int down(const void* h, const int32_t* offsets, int64_t rows_total, int64_t max_rows, int64_t E,
         int64_t H, int64_t I, const void* blocks, const void* scales, const void* bias,
         int bias_dtype, void* y, int algo, cudaStream_t st) {
  BS_TRY(check_expert_args("bs_moe_down", h, blocks, scales, y, rows_total, E, I, H, bias_dtype,
                           algo));
  BS_ARG(offsets, "bs_moe_down: null expert_offsets");
  if (rows_total == 0) return BS_OK;
  BS_TRY(check_device());
  const int a = pick_algo(algo, rows_total, E, scales, I, H);
  const int bf32 = bias_dtype == BS_F32;
  if (a == BS_ALGO_GEMV)
    return gemv_plain_launch(h, offsets, rows_total, E, I, H, blocks, scales, bias, bf32, y, st);
  auto launch = a == BS_ALGO_TCGEN05_PAIR ? tc_pair_launch : tc_grouped_launch;
  return launch(1, h, offsets, rows_total, max_rows, E, I, H, blocks, scales, bias, bf32, 0.f, 0.f, y, st);
}

struct Workspace {
  void* router;
  size_t router_bytes;
  void* dispatch;
  size_t dispatch_bytes;
  int32_t* offsets;
  int32_t* row_of_slot;
  int32_t* token_of_row;
  void* x_perm;
  void* h;
  void* y;
  size_t total;
};

Workspace carve(void* base, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  Workspace w{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return base ? static_cast<char*>(base) + at : nullptr;
  };
  const int64_t S = T * k;
  // sized for an fp32 router (the larger split); a bf16 router uses less
  w.router_bytes = router_workspace_bytes(T, H, E, BS_F32);
  w.router = take(w.router_bytes);
  w.dispatch_bytes = dispatch_workspace_bytes(T, k, E);
  w.dispatch = take(w.dispatch_bytes);
  w.offsets = reinterpret_cast<int32_t*>(take((size_t)(E + 1) * sizeof(int32_t)));
  w.row_of_slot = reinterpret_cast<int32_t*>(take((size_t)S * sizeof(int32_t)));
  w.token_of_row = reinterpret_cast<int32_t*>(take((size_t)S * sizeof(int32_t)));
  w.x_perm = take((size_t)S * H * 2);
  w.h = take((size_t)S * I * 2);
  w.y = take((size_t)S * H * 2);
  w.total = o;
  return w;
}

}  // namespace bs

extern "C" int bs_moe_gate_up(const void* x_perm, const int32_t* expert_offsets, int64_t rows_total,
                              int64_t max_rows_per_expert, int64_t E, int64_t H, int64_t I,
                              const void* blocks, const void* scales, const void* bias,
                              int bias_dtype, float alpha, float limit, void* h, int algo,
                              void* stream) {
  return bs::gate_up(x_perm, expert_offsets, rows_total, max_rows_per_expert, E, H, I, blocks,
                     scales, bias, bias_dtype, alpha, limit, h, algo,
                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int bs_moe_down(const void* h, const int32_t* expert_offsets, int64_t rows_total,
                           int64_t max_rows_per_expert, int64_t E, int64_t H, int64_t I,
                           const void* blocks, const void* scales, const void* bias, int bias_dtype,
                           void* y, int algo, void* stream) {
  return bs::down(h, expert_offsets, rows_total, max_rows_per_expert, E, H, I, blocks, scales, bias,
                  bias_dtype, y, algo, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int bs_mxfp4_matmul(const void* x, int64_t m, int64_t K, const void* blocks,
                               const void* scales, int64_t N, const void* bias, void* out, int algo,
                               void* stream) {
  using namespace bs;
  BS_TRY(check_expert_args("bs_mxfp4_matmul", x, blocks, scales, out, m, 1, K, N, BS_BF16, algo));
  if (m == 0) return BS_OK;
  BS_TRY(check_device());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int a = pick_algo(algo, m, 1, scales, K, N);
  if (a == BS_ALGO_GEMV)
    return gemv_plain_launch(x, nullptr, m, 1, K, N, blocks, scales, bias, 0, out, st);
  auto launch = a == BS_ALGO_TCGEN05_PAIR ? tc_pair_launch : tc_grouped_launch;
  return launch(1, x, nullptr, m, m, 1, K, N, blocks, scales, bias, 0, 0.f, 0.f, out, st);
}

namespace bs {
namespace {
size_t moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  size_t n = carve(nullptr, T, H, I, E, k).total;
  if (decode_supported(T, H, I, E, k)) n = std::max(n, decode_workspace_bytes(T, H, I, E, k));
  if (T >= 1 && T <= 8 && k <= 8 && E <= 1024) n = std::max(n, fused_workspace_bytes(T, H, I, E, k));
  return n;
}
}  // namespace
}  // namespace bs

extern "C" size_t bs_moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return bs::moe_workspace_bytes(T, H, I, E, k);
}

namespace bs {
namespace {
// The layer; with residual != NULL the combine also adds it (bf16 + bf16).
int moe_forward_impl(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                     const void* router_weight, const void* router_bias, int router_dtype,
                     float* scores, int32_t* indices, const void* gate_up_blocks,
                     const void* gate_up_scales, const void* gate_up_bias,
                     const void* down_blocks, const void* down_scales,
                     const void* down_bias, int bias_dtype, float alpha, float limit,
                     void* out, void* workspace, size_t workspace_bytes, int algo,
                     void* stream, const void* residual) {
  BS_ARG(x && scores && indices && out, "bs_moe_forward: null pointer");
  BS_ARG(T >= 0 && H > 0 && I > 0 && E > 0 && k > 0 && k <= E, "bs_moe_forward: bad sizes");
  BS_ARG((router_weight == nullptr) == (router_bias == nullptr),
         "bs_moe_forward: router weight and bias go together");
  BS_ARG(algo >= BS_ALGO_AUTO && algo <= BS_ALGO_TCGEN05_PAIR, "bs_moe_forward: unknown algo %d", algo);
  if (T == 0) return BS_OK;
  BS_ARG(workspace, "bs_moe_forward: null workspace");
  BS_ALIGNED16(workspace, "workspace");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // the single-launch decode kernel runs on request only: measured with the
  // weights cold and the code cached (a model's layer loop), the four-launch
  // block-scaled path below is faster at every T it takes
  if (algo == BS_ALGO_FUSED) {
    BS_ARG(router_dtype == BS_F32 || router_dtype == BS_BF16 || !router_weight,
           "bs_moe_forward: router dtype must be bf16 or f32");
    BS_ARG(bias_dtype == BS_BF16 || bias_dtype == BS_F32, "bs_moe_forward: bias dtype must be bf16 or f32");
    BS_ARG(T <= 8 && k <= 8 && E <= 1024, "bs_moe_forward: BS_ALGO_FUSED needs T <= 8, k <= 8, E <= 1024");
    const size_t need = fused_workspace_bytes(T, H, I, E, k);
    BS_REQUIRE(workspace_bytes >= need, BS_ERR_CAPACITY,
               "bs_moe_forward: workspace of %zu bytes is smaller than the %zu needed", workspace_bytes, need);
    BS_TRY(check_device());
    NvtxRange r("bs.fused_decode_layer");
    return fused_forward(x, T, H, I, E, k, router_weight, router_bias, router_dtype, scores, indices,
                         gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks, down_scales, down_bias,
                         bias_dtype == BS_F32, alpha, limit, out, workspace, st, residual);
  }
  // AUTO takes the decode path whenever it applies (T <= 64, aligned blocks).
  const bool mx = algo == BS_ALGO_MX ||
                  (algo == BS_ALGO_AUTO && decode_supported(T, H, I, E, k) &&
                   ((uintptr_t)gate_up_blocks | (uintptr_t)down_blocks | (uintptr_t)gate_up_scales |
                    (uintptr_t)down_scales) % 16 == 0);
  if (mx) {
    BS_ARG(decode_supported(T, H, I, E, k),
           "bs_moe_forward: BS_ALGO_MX needs T <= 64, H and I multiples of 64, E <= 1024, k <= 32");
    BS_ARG(router_dtype == BS_F32 || router_dtype == BS_BF16 || !router_weight,
           "bs_moe_forward: router dtype must be bf16 or f32");
    BS_ARG(bias_dtype == BS_BF16 || bias_dtype == BS_F32, "bs_moe_forward: bias dtype must be bf16 or f32");
    const size_t need = decode_workspace_bytes(T, H, I, E, k);
    BS_REQUIRE(workspace_bytes >= need, BS_ERR_CAPACITY,
               "bs_moe_forward: workspace of %zu bytes is smaller than the %zu needed", workspace_bytes,
               need);
    BS_TRY(check_device());
    NvtxRange r("bs.decode_layer");
    return decode_forward(x, T, H, I, E, k, router_weight, router_bias, router_dtype, scores, indices,
                          gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks, down_scales,
                          down_bias, bias_dtype == BS_F32, alpha, limit, out, workspace, st, residual);
  }
  const Workspace w = carve(workspace, T, H, I, E, k);
  BS_REQUIRE(workspace_bytes >= w.total, BS_ERR_CAPACITY,
             "bs_moe_forward: workspace of %zu bytes is smaller than the %zu needed",
             workspace_bytes, w.total);
  NvtxRange layer_range("bs.layer");
  if (router_weight) {
    NvtxRange r("bs.router");
    BS_TRY(router_launch(x, BS_BF16, router_weight, router_bias, router_dtype, T, H, E, k, nullptr,
                         scores, indices, BS_I32, w.router, w.router_bytes, st));
  }
  {
    NvtxRange r("bs.dispatch");
    BS_TRY(dispatch_launch(indices, BS_I32, T, k, E, x, H, w.offsets, w.row_of_slot, w.token_of_row,
                         w.x_perm, w.dispatch, w.dispatch_bytes, st));
  }
  const int64_t S = T * k;
  {
    NvtxRange r("bs.gate_up");
    BS_TRY(gate_up(w.x_perm, w.offsets, S, S, E, H, I, gate_up_blocks, gate_up_scales, gate_up_bias,
                 bias_dtype, alpha, limit, w.h, algo, st));
  }
  {
    NvtxRange r("bs.down");
    BS_TRY(down(w.h, w.offsets, S, S, E, H, I, down_blocks, down_scales, down_bias, bias_dtype, w.y,
              algo, st));
  }
  NvtxRange r("bs.combine");
  BS_TRY(combine_launch(w.y, w.row_of_slot, scores, T, k, H, out, st, residual));
  return BS_OK;
}
}  // namespace
}  // namespace bs

extern "C" int bs_moe_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                              const void* router_weight, const void* router_bias, int router_dtype,
                              float* scores, int32_t* indices, const void* gate_up_blocks,
                              const void* gate_up_scales, const void* gate_up_bias,
                              const void* down_blocks, const void* down_scales,
                              const void* down_bias, int bias_dtype, float alpha, float limit,
                              void* out, void* workspace, size_t workspace_bytes, int algo,
                              void* stream) {
  return bs::moe_forward_impl(x, T, H, I, E, k, router_weight, router_bias, router_dtype, scores, indices,
                              gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks, down_scales, down_bias,
                              bias_dtype, alpha, limit, out, workspace, workspace_bytes, algo, stream, nullptr);
}

extern "C" int bs_moe_decode(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                             const void* router_weight, const void* router_bias, int router_dtype,
                             float* scores, int32_t* indices, const void* gate_up_blocks,
                             const void* gate_up_scales, const void* gate_up_bias,
                             const void* down_blocks, const void* down_scales, const void* down_bias,
                             int bias_dtype, float alpha, float limit, void* out, void* workspace,
                             size_t workspace_bytes, void* stream) {
  return bs::moe_forward_impl(x, T, H, I, E, k, router_weight, router_bias, router_dtype, scores, indices,
                              gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks, down_scales, down_bias,
                              bias_dtype, alpha, limit, out, workspace, workspace_bytes, BS_ALGO_MX, stream,
                              nullptr);
}

extern "C" size_t bs_moe_block_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t k) {
  return bs::align_up(bs_moe_workspace_bytes(T, H, I, E, k), 256) + bs::align_up((size_t)T * H * 2, 256);
}

extern "C" int bs_moe_block_forward(const void* x, int64_t T, int64_t H, int64_t I, int64_t E, int64_t k,
                                    const void* norm_weight, int norm_dtype, float eps,
                                    const void* router_weight, const void* router_bias, int router_dtype,
                                    float* scores, int32_t* indices, const void* gate_up_blocks,
                                    const void* gate_up_scales, const void* gate_up_bias,
                                    const void* down_blocks, const void* down_scales, const void* down_bias,
                                    int bias_dtype, float alpha, float limit, void* out, void* workspace,
                                    size_t workspace_bytes, int algo, void* stream) {
  using namespace bs;
  BS_ARG(x && norm_weight && out && workspace, "bs_moe_block_forward: null pointer");
  BS_ARG(out != x, "bs_moe_block_forward: out must not alias x (x is the residual)");
  BS_ARG(T >= 0 && H > 0, "bs_moe_block_forward: bad sizes");
  if (T == 0) return BS_OK;
  const size_t layer_ws = align_up(bs_moe_workspace_bytes(T, H, I, E, k), 256);
  BS_REQUIRE(workspace_bytes >= bs_moe_block_workspace_bytes(T, H, I, E, k), BS_ERR_CAPACITY,
             "bs_moe_block_forward: workspace of %zu bytes is smaller than the %zu needed", workspace_bytes,
             bs_moe_block_workspace_bytes(T, H, I, E, k));
  void* xn = static_cast<char*>(workspace) + layer_ws;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  BS_TRY(rmsnorm_launch(x, T, H, norm_weight, norm_dtype, eps, xn, st));
  return moe_forward_impl(xn, T, H, I, E, k, router_weight, router_bias, router_dtype, scores, indices,
                          gate_up_blocks, gate_up_scales, gate_up_bias, down_blocks, down_scales, down_bias,
                          bias_dtype, alpha, limit, out, workspace, layer_ws, algo, stream, x);
}
