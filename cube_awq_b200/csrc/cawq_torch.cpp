// cawq_torch.cpp — compiled host path of the module forward (torch binding).
//
// AWQGEMMLinear.forward (src/modules/awq_gemm.rs:146-232) is called once per
// layer per token; at decode sizes its host work is of the order of the
// kernel's own device time. This extension holds a layer's tensors and the
// constant arguments of its cawq_gemm call, and its forward does, in C++: the
// input checks, one allocation of the output through torch's caching
// allocator on the input's device, the current stream, and the C call. The
// Python module keeps the reference's API and messages: whenever an input
// does not fit (wrong dtype, device, rank, K, layout), forward returns None
// and the module takes its general path, which raises the reference's errors.
//
// Nothing here computes: the kernels are libcube_awq.so's.
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include "cube_awq.h"

namespace {

struct Layer {
  at::Tensor qweight, qzeros, scales, bias;  // held, so their storage stays alive
  const uint32_t* qw = nullptr;
  const uint32_t* qz = nullptr;
  const void* sc = nullptr;
  const void* b = nullptr;
  int64_t k = 0, n = 0, g = 0;
  c10::ScalarType dtype = c10::ScalarType::Float;
  cawq_dtype code = CAWQ_F32;
  cawq_order order = CAWQ_ORDER_AWQ;
  c10::DeviceIndex device = 0;

  Layer(at::Tensor qweight_, at::Tensor qzeros_, at::Tensor scales_,
        c10::optional<at::Tensor> bias_, int64_t group_size, int64_t order_)
      : qweight(std::move(qweight_)), qzeros(std::move(qzeros_)), scales(std::move(scales_)) {
    TORCH_CHECK(qweight.is_cuda() && qzeros.is_cuda() && scales.is_cuda(),
                "layer tensors must be on a GPU");
    TORCH_CHECK(qweight.is_contiguous() && qzeros.is_contiguous() && scales.is_contiguous(),
                "layer tensors must be contiguous");
    TORCH_CHECK(qweight.dim() == 2 && scales.dim() == 2, "qweight and scales must be 2-D");
    if (bias_.has_value()) {
      bias = *bias_;
      TORCH_CHECK(bias.is_cuda() && bias.is_contiguous() && bias.scalar_type() == scales.scalar_type(),
                  "bias must be a contiguous GPU tensor in the scales' dtype");
      b = bias.data_ptr();
    }
    dtype = scales.scalar_type();
    switch (dtype) {
      case c10::ScalarType::Float: code = CAWQ_F32; break;
      case c10::ScalarType::Half: code = CAWQ_F16; break;
      case c10::ScalarType::BFloat16: code = CAWQ_BF16; break;
      default: TORCH_CHECK(false, "scales must be float32, float16 or bfloat16");
    }
    order = order_ == 1 ? CAWQ_ORDER_NATURAL : CAWQ_ORDER_AWQ;
    k = qweight.size(0);
    n = qweight.size(1) * 8;
    g = group_size;
    device = scales.get_device();
    qw = static_cast<const uint32_t*>(qweight.data_ptr());
    qz = static_cast<const uint32_t*>(qzeros.data_ptr());
    sc = scales.data_ptr();
  }

  // out = x · deq(W) (+ bias) for a contiguous [rows, K] input of the layer's
  // dtype on its device; None for any other input (the caller's general path
  // then checks it and raises); an int status if the C call failed.
  py::object forward(const at::Tensor& x) const {
    if (!x.is_cuda() || x.dim() != 2 || x.scalar_type() != dtype || x.get_device() != device ||
        x.size(1) != k || !x.is_contiguous())
      return py::none();
    const int64_t rows = x.size(0);
    at::Tensor out = at::empty({rows, n}, x.options());
    if (rows == 0) return py::cast(out);
    cudaStream_t s = c10::cuda::getCurrentCUDAStream(device).stream();
    const cawq_status st = cawq_gemm(x.data_ptr(), qw, qz, sc, b, out.data_ptr(),
                                     static_cast<size_t>(rows), static_cast<size_t>(k),
                                     static_cast<size_t>(n), static_cast<size_t>(g), code, code,
                                     order, static_cast<size_t>(n), s);
    if (st != CAWQ_OK) return py::int_(static_cast<int>(st));
    return py::cast(out);
  }
};

}  // namespace

PYBIND11_MODULE(_cawq_torch, m) {
  m.doc() = "compiled host path of the cube_awq_b200 module forward";
  py::class_<Layer>(m, "Layer")
      .def(py::init<at::Tensor, at::Tensor, at::Tensor, c10::optional<at::Tensor>, int64_t,
                    int64_t>(),
           py::arg("qweight"), py::arg("qzeros"), py::arg("scales"), py::arg("bias"),
           py::arg("group_size"), py::arg("order"))
      .def("forward", &Layer::forward);
}
