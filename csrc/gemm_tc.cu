// Host entry of the tcgen05 GEMM: argument checks, tensor-map encoding and
// dispatch to the instantiation for the requested tile width / epilogue.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <algorithm>
#include <mutex>

#include "gemm_tc.cuh"

namespace gb {

bool& pdl_enabled() {
  // Off by default: on the decode loop (captured in a CUDA graph) it measured
  // slower than plain stream order.  _C.set_pdl(True) turns it on for measurements.
  static bool on = false;
  return on;
}



using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Tensor map for a row-major bf16 matrix [rows, cols] with row stride `ld`
// elements, loaded in boxes of [box_rows, 64] with the 128-byte swizzle.
CUtensorMap make_tmap_bf16(const void* ptr, long rows, long cols, long ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return map;
}

static void check_operand(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kBFloat16, name, " must be a CUDA bf16 tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with unit inner stride");
}

// Generic entry: see module docstring for the meaning of each epilogue.
void gemm_tc(torch::Tensor A, torch::Tensor B, c10::optional<torch::Tensor> A2,
             c10::optional<torch::Tensor> B2, torch::Tensor C, c10::optional<torch::Tensor> R,
             c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> targets,
             c10::optional<torch::Tensor> tgt_logit, c10::optional<torch::Tensor> row_lse,
             c10::optional<torch::Tensor> row_scale, int64_t epilogue, bool swap, int64_t bn,
             int64_t splits, torch::Tensor err, int64_t max_ctas, c10::optional<torch::Tensor> push_dst,
             c10::optional<torch::Tensor> push_flag, c10::optional<torch::Tensor> tile_ctr, int64_t layout,
             c10::optional<torch::Tensor> push_out, c10::optional<torch::Tensor> push_sig, int64_t push_self,
             int64_t push_rows, int64_t push_fence_once) {
  check_operand(A, "A");
  check_operand(B, "B");
  // layout bit 1: A given as [K, M] (MN-major); bit 0: B given as [K, N]
  const bool a_mn = (layout & 2) != 0, b_mn = (layout & 1) != 0;
  const int64_t Ka = a_mn ? A.size(0) : A.size(1), Kb = b_mn ? B.size(0) : B.size(1);
  const int64_t Mdim = a_mn ? A.size(1) : A.size(0), Ndim = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK(Ka == Kb, "A and B must share K");
  TORCH_CHECK(!b_mn || bn % 64 == 0, "MN-major B needs an N tile that is a multiple of 64");
  // K need not be a multiple of 64: TMA zero-fills the tail of the last K-block.
  const c10::cuda::CUDAGuard guard(A.device());
  const int device = A.get_device();
  GemmArgs args{};
  args.M = static_cast<int>(Mdim);
  args.N = static_cast<int>(Ndim);
  args.kb_main = static_cast<int>((Ka + BK - 1) / BK);
  args.kb_ext = 0;
  args.splits = static_cast<int>(std::max<int64_t>(splits, 1));
  args.C = C.data_ptr();
  args.ldc = C.stride(0);
  args.err = err.data_ptr<int>();
  const int box_a = BM;
  const int box_b = static_cast<int>(bn);
  // MN-major operands are loaded as [64 K-rows, 64 MN] boxes
  CUtensorMap ta = a_mn ? make_tmap_bf16(A.data_ptr(), A.size(0), A.size(1), A.stride(0), 64)
                        : make_tmap_bf16(A.data_ptr(), A.size(0), A.size(1), A.stride(0), box_a);
  CUtensorMap tb = b_mn ? make_tmap_bf16(B.data_ptr(), B.size(0), B.size(1), B.stride(0), 64)
                        : make_tmap_bf16(B.data_ptr(), B.size(0), B.size(1), B.stride(0), box_b);
  CUtensorMap ta2 = ta, tb2 = tb;
  if (A2.has_value() && A2->defined()) {
    TORCH_CHECK(B2.has_value() && B2->defined(), "A2 requires B2");
    check_operand(*A2, "A2");
    check_operand(*B2, "B2");
    const int64_t K2a = a_mn ? A2->size(0) : A2->size(1), K2b = b_mn ? B2->size(0) : B2->size(1);
    const int64_t M2 = a_mn ? A2->size(1) : A2->size(0), N2 = b_mn ? B2->size(1) : B2->size(0);
    TORCH_CHECK(K2a == K2b, "extension K must match");
    TORCH_CHECK(M2 == Mdim && N2 == Ndim, "extension operands must match M and N");
    args.kb_ext = static_cast<int>((K2a + BK - 1) / BK);
    ta2 = a_mn ? make_tmap_bf16(A2->data_ptr(), A2->size(0), A2->size(1), A2->stride(0), 64)
               : make_tmap_bf16(A2->data_ptr(), A2->size(0), A2->size(1), A2->stride(0), box_a);
    tb2 = b_mn ? make_tmap_bf16(B2->data_ptr(), B2->size(0), B2->size(1), B2->stride(0), 64)
               : make_tmap_bf16(B2->data_ptr(), B2->size(0), B2->size(1), B2->stride(0), box_b);
  }
  if (R.has_value() && R->defined()) {
    args.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    args.ldr = R->stride(0);
  }
  if (aux.has_value() && aux->defined()) {
    args.aux = aux->data_ptr();
    args.ldaux = aux->stride(0);
    if (epilogue == kLSE) args.ldaux = aux->stride(0) / 2;  // float2 units
  }
  if (targets.has_value() && targets->defined()) args.targets = targets->data_ptr<int64_t>();
  if (tgt_logit.has_value() && tgt_logit->defined()) args.tgt_logit = tgt_logit->data_ptr<float>();
  if (row_lse.has_value() && row_lse->defined()) args.row_lse = row_lse->data_ptr<float>();
  if (row_scale.has_value() && row_scale->defined()) args.row_scale = row_scale->data_ptr<float>();
  if (epilogue == kLSE || epilogue == kSoftmaxGrad)
    TORCH_CHECK(args.targets != nullptr, "log-prob epilogues need targets");
  if (epilogue == kLSE) TORCH_CHECK(args.tgt_logit != nullptr && args.aux != nullptr, "LSE epilogue needs aux and tgt_logit");
  if (epilogue == kSoftmaxGrad) TORCH_CHECK(args.row_lse != nullptr && args.row_scale != nullptr, "softmax-grad epilogue needs lse and scale");
  const bool split_swiglu = epilogue == kSwiGLU && swap && args.splits > 1;
  TORCH_CHECK(epilogue == kAtomicF32 || args.splits == 1 || split_swiglu,
              "split-K requires the atomic epilogue (or the swap SwiGLU epilogue with a workspace)");
  {
    const int kb_total = args.kb_main + args.kb_ext;
    const int per = (kb_total + args.splits - 1) / args.splits;
    args.nonempty_splits = (kb_total + per - 1) / per;
  }
  if (split_swiglu) {
    TORCH_CHECK(args.splits <= 4, "split-K SwiGLU supports at most 4 splits");
    // Only the tiles of the persistent grid's last (partial) wave are split: the
    // first full waves run whole-K tiles with the SwiGLU epilogue directly.
    const int tiles = static_cast<int>(((Mdim + BM - 1) / BM) * ((Ndim + bn - 1) / bn));
    int ctas = num_sms(device);
    if (max_ctas > 0) ctas = std::min<int>(ctas, static_cast<int>(max_ctas));
    const int full = tiles / ctas * ctas;
    const int rem = tiles - full;
    args.full_tiles = full;
    args.splits = rem == 0 ? 1 : std::max(1, std::min(args.splits, ctas / rem));
    if (args.splits == 1) args.full_tiles = 0;
    {
      const int kb_total = args.kb_main + args.kb_ext;
      const int per = (kb_total + args.splits - 1) / args.splits;
      args.nonempty_splits = (kb_total + per - 1) / per;
    }
    TORCH_CHECK(aux.has_value() && aux->defined() && aux->scalar_type() == torch::kFloat32 && aux->is_contiguous() &&
                    aux->numel() >= static_cast<int64_t>(args.splits) * Mdim * Ndim,
                "split-K SwiGLU needs an fp32 workspace of splits x tokens x features");
    TORCH_CHECK(tile_ctr.has_value() && tile_ctr->defined() && tile_ctr->scalar_type() == torch::kInt32 &&
                    tile_ctr->numel() >= ((Mdim + BM - 1) / BM) * ((Ndim + bn - 1) / bn),
                "split-K SwiGLU needs a zeroed int32 tile counter per output tile");
    TORCH_CHECK(layout == 0, "split-K SwiGLU takes K-major operands");
    args.ldaux = Mdim;
    args.tile_ctr = tile_ctr->data_ptr<int>();
  }
  if (push_dst.has_value() && push_dst->defined()) {
    TORCH_CHECK(swap && epilogue == kAtomicF32, "tile push needs the swap atomic epilogue");
    TORCH_CHECK(push_flag.has_value() && tile_ctr.has_value(), "tile push needs flags and tile counters");
    TORCH_CHECK(push_dst->device().is_cpu() && push_dst->scalar_type() == torch::kInt64 &&
                    push_flag->device().is_cpu() && push_flag->scalar_type() == torch::kInt64 &&
                    push_dst->numel() == push_flag->numel() && push_dst->numel() <= kMaxPeers,
                "push_dst / push_flag: CPU int64 address tables of equal length <= 8");
    const int np = static_cast<int>(push_dst->numel());
    auto pd = push_dst->contiguous();
    auto pf = push_flag->contiguous();
    for (int q = 0; q < np; ++q) {
      args.push_dst[q] = reinterpret_cast<float*>(pd.data_ptr<int64_t>()[q]);
      args.push_flag[q] = reinterpret_cast<int*>(pf.data_ptr<int64_t>()[q]);
    }
    args.npeers = np;
    const int num_tiles = static_cast<int>(((Mdim + BM - 1) / BM) * ((Ndim + bn - 1) / bn));
    TORCH_CHECK(tile_ctr->scalar_type() == torch::kInt32 && tile_ctr->is_cuda() && tile_ctr->numel() >= num_tiles,
                "tile_ctr must be a zeroed int32 CUDA tensor with one entry per output tile");
    args.tile_ctr = tile_ctr->data_ptr<int>();
    TORCH_CHECK(layout == 0 && C.scalar_type() == torch::kFloat32 && C.size(0) == Ndim && C.size(1) == Mdim,
                "tile push writes C [tokens, features] in full");
  }
  if (push_out.has_value() && push_out->defined()) {
    // fused all-reduce / reduce-scatter of a non-swap bf16 GEMM: C only supplies the row stride
    TORCH_CHECK(!swap && epilogue == kStoreBF16 && (layout == 0 || layout == 1),
                "slot push needs the non-swap bf16 store epilogue with a K-major A");
    TORCH_CHECK(C.scalar_type() == torch::kBFloat16 && C.stride(1) == 1 && C.stride(0) >= Ndim &&
                    (C.stride(0) * 2) % 16 == 0 && Ndim % 8 == 0,
                "slot push: bf16 slots with 16-byte aligned rows and N a multiple of 8");
    TORCH_CHECK(push_sig.has_value() && push_sig->defined(), "slot push needs arrival counters");
    TORCH_CHECK(push_out->device().is_cpu() && push_out->scalar_type() == torch::kInt64 &&
                    push_sig->device().is_cpu() && push_sig->scalar_type() == torch::kInt64 &&
                    push_out->numel() == push_sig->numel() && push_out->numel() >= 1 && push_out->numel() <= kMaxPeers,
                "push_out / push_sig: CPU int64 address tables of equal length in [1, 8]");
    const int np = static_cast<int>(push_out->numel());
    TORCH_CHECK(push_self >= 0 && push_self < np, "push_self must index the address tables");
    TORCH_CHECK(push_rows == 0 || static_cast<int64_t>(push_rows) * np == Mdim,
                "reduce-scatter push needs rows = M / ranks");
    auto po = push_out->contiguous();
    auto ps = push_sig->contiguous();
    for (int q = 0; q < np; ++q) {
      args.out_push[q] = reinterpret_cast<__nv_bfloat16*>(po.data_ptr<int64_t>()[q]);
      args.sig_push[q] = reinterpret_cast<unsigned long long*>(ps.data_ptr<int64_t>()[q]);
      TORCH_CHECK(args.out_push[q] != nullptr && reinterpret_cast<uintptr_t>(args.out_push[q]) % 16 == 0,
                  "slot push: 16-byte aligned destination slots");
    }
    args.npush = np;
    args.push_self = static_cast<int>(push_self);
    args.push_rows = static_cast<int>(push_rows);
    args.push_fence_once = push_fence_once ? 1 : 0;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  const int mc = static_cast<int>(max_ctas);
  TORCH_CHECK(!swap || (epilogue != kLSE && epilogue != kSoftmaxGrad), "log-prob epilogues are not available in swap mode");
  GemmLauncher fn = nullptr;
  if (layout != 0) {
    fn = gemm_launcher_mn(static_cast<int>(bn), static_cast<int>(epilogue), swap, static_cast<int>(layout));
  } else if (swap) {
    fn = gemm_launcher_swap(static_cast<int>(bn), static_cast<int>(epilogue));
  } else if (bn == 256) {
    fn = gemm_launcher_n256(static_cast<int>(epilogue));
  } else if (bn == 128) {
    fn = gemm_launcher_n128(static_cast<int>(epilogue));
  } else if (bn == 64) {
    fn = gemm_launcher_n64(static_cast<int>(epilogue));
  }
  TORCH_CHECK(fn != nullptr, "no GEMM instantiation for bn=", bn, " swap=", swap, " epilogue=", epilogue,
              " layout=", layout);
  fn(ta, tb, ta2, tb2, args, mc, stream, device);
}

}  // namespace gb
