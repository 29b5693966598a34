// Definitions for the reference's GPU entry points whose sources are absent
// from the reference tree (exl3_gemv.cu, p2b_batched.cu, exl3_gemm.cu) or need
// exllamav3 headers that are absent (p2b_moe.cu, lna_moe_decode.cu,
// lna_moe_ticket.cu).  Each raises: the CPU build of the reference's
// bindings.cpp only serves dequant_trellis and the CPU branch of exl3_gemv.
#include <torch/extension.h>
#include <vector>

#define ABSENT(name) TORCH_CHECK(false, name " is not part of the CPU reference build")

at::Tensor exl3_gemv_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&, int64_t, bool, int64_t) { ABSENT("exl3_gemv_cuda"); }
at::Tensor exl3_gemm_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&, int64_t, bool) { ABSENT("exl3_gemm_cuda"); }
at::Tensor p2b_gemv_batched_cuda(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const at::Tensor&, const at::Tensor&, int64_t, bool,
                                 int64_t) { ABSENT("p2b_gemv_batched_cuda"); }
at::Tensor p2b_fused_moe_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const at::Tensor&, int64_t, int64_t, int64_t, bool,
                              double) { ABSENT("p2b_fused_moe_cuda"); }
at::Tensor lna_moe_decode_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&,
                               const at::Tensor&, const at::Tensor&, const at::Tensor&,
                               const at::Tensor&, const at::Tensor&, const at::Tensor&,
                               const at::Tensor&, const at::Tensor&, const at::Tensor&,
                               const at::Tensor&, int64_t, double,
                               const at::Tensor&) { ABSENT("lna_moe_decode_cuda"); }
int64_t lna_moe_scratch_bytes_cuda() { ABSENT("lna_moe_scratch_bytes_cuda"); }
void lna_moe_prepare_cuda(int64_t, int64_t) { ABSENT("lna_moe_prepare_cuda"); }
std::vector<int64_t> lna_moe_info_cuda(int64_t, int64_t) { ABSENT("lna_moe_info_cuda"); }
at::Tensor lna2_moe_decode_cuda(const at::Tensor&, at::Tensor&, const at::Tensor&,
                                const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                const at::Tensor&, int64_t, double,
                                const at::Tensor&) { ABSENT("lna2_moe_decode_cuda"); }
int64_t lna2_moe_scratch_bytes_cuda() { ABSENT("lna2_moe_scratch_bytes_cuda"); }
int64_t lna2_moe_max_rows_cuda() { ABSENT("lna2_moe_max_rows_cuda"); }
void lna2_moe_prepare_cuda(int64_t) { ABSENT("lna2_moe_prepare_cuda"); }
std::vector<int64_t> lna2_moe_info_cuda(int64_t) { ABSENT("lna2_moe_info_cuda"); }
