// Minimal ATen/c10 includes for the host-side launch wrappers inside .cu files
// (torch/extension.h pulls in pybind11 and the Python API; this keeps nvcc fast).
#pragma once
#include <ATen/core/Tensor.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/cuda/CUDAException.h>
#include <c10/util/Exception.h>
#include <c10/util/Optional.h>

namespace at { namespace cuda { using c10::cuda::getCurrentCUDAStream; } }
namespace torch { using at::Tensor; }

static inline void* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr() : nullptr;
}
