// Stand-in for a header that is absent from the reference tree
// (recipe-lna/lna2/setup.py:25-31 lists its .cu, which is not shipped).
// It only declares the GPU entry that bindings.cpp names; the CPU path
// (dequant_cpu + at::mm) never calls it.  Built into oracle/_ref/ only.
#pragma once
#include <torch/extension.h>
at::Tensor p2b_gemv_batched_cuda(const at::Tensor& x, const at::Tensor& trellis_ptrs,
                                 const at::Tensor& suh_ptrs, const at::Tensor& svh_ptrs,
                                 const at::Tensor& expert_indices, int64_t bits,
                                 bool mcg, int64_t mmode);
