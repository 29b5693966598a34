// Stand-in for a header that is absent from the reference tree (see
// p2b_batched.cuh in this folder).  Declares the GPU entry bindings.cpp names.
#pragma once
#include <torch/extension.h>
at::Tensor exl3_gemm_cuda(const at::Tensor& x, const at::Tensor& trellis,
                          const at::Tensor& suh, const at::Tensor& svh,
                          int64_t bits, bool mcg);
