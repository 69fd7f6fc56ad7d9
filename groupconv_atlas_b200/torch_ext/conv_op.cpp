// PyTorch front end of gc_cuda_conv for the torch.nn module: allocates the
// output with PyTorch's caching allocator and calls the C ABI on the current
// CUDA stream, all in C++, so that a substituted layer costs about as much
// host time per call as a cuDNN convolution.  The descriptors are built
// exactly as the reference's Python caller builds them (bench/api.py:71-83):
// element strides, the tensor's device and device index, float32 or float64.
// Errors come back as gc_status values with the library's thread-local
// message; nothing here computes a convolution.  conv_ex does the same for
// gc_b200_conv_ex (bias, activation, channels-last output).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <stdexcept>
#include <string>

#include "groupconv.h"

namespace {

gc_tensor describe(const at::Tensor &t) {
    gc_tensor d{};
    d.data = t.data_ptr();
    d.bytes = static_cast<uint64_t>(t.numel()) * t.element_size();
    d.dtype = t.scalar_type() == at::kFloat ? GC_F32 : t.scalar_type() == at::kDouble ? GC_F64 : -1;
    d.device = t.is_cuda() ? GC_CUDA : t.is_cpu() ? GC_CPU : -1;
    d.device_index = t.is_cuda() ? t.get_device() : 0;
    d.rank = static_cast<int32_t>(t.dim());
    for (int i = 0; i < 4 && i < t.dim(); ++i) {
        d.dims[i] = t.size(i);
        d.strides[i] = t.stride(i);
    }
    return d;
}

// y = conv(x, w) with the layer's geometry; x must be 4-D.  Raises
// RuntimeError("gc_status <s>: <message>") on any non-OK status.
at::Tensor conv(const at::Tensor &x, const at::Tensor &w, int64_t cout, int64_t r, int64_t s, int64_t groups,
                int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw, int64_t implementation) {
    if (x.dim() != 4) throw std::invalid_argument("input must be 4-D NCHW");
    const gc_shape p{x.size(0), x.size(1), cout, x.size(2), x.size(3), r, s, groups, sh, sw, ph, pw, dh, dw};
    int64_t ho = 0, wo = 0;
    int st = gc_validate_shape(&p, &ho, &wo);
    if (st != GC_OK) throw std::runtime_error("gc_status " + std::to_string(st) + ": " + gc_last_error());
    // gc_cuda_conv requires the tensors' device to be the current device (as
    // nn.Conv2d runs on its input's device whatever the current one is).
    c10::OptionalDeviceGuard guard;
    if (x.is_cuda()) guard.reset_device(x.device());
    at::Tensor y = at::empty({p.n, cout, ho, wo}, x.options());
    const gc_tensor xd = describe(x), wd = describe(w);
    gc_tensor yd = describe(y);
    void *stream = x.is_cuda() ? static_cast<void *>(c10::cuda::getCurrentCUDAStream(x.get_device()).stream())
                               : nullptr;
    st = gc_cuda_conv(&p, &xd, &wd, &yd, static_cast<int>(implementation), stream);
    if (st != GC_OK) throw std::runtime_error("gc_status " + std::to_string(st) + ": " + gc_last_error());
    return y;
}

// y = act(conv(x, w) + bias) through gc_b200_conv_ex: bias optional, layout
// 0 (NCHW output) or 1 (channels-last output), activation GC_B200_ACT_*.
at::Tensor conv_ex(const at::Tensor &x, const at::Tensor &w, const c10::optional<at::Tensor> &bias, int64_t cout,
                   int64_t r, int64_t s, int64_t groups, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                   int64_t dw, int64_t layout, int64_t activation) {
    if (x.dim() != 4) throw std::invalid_argument("input must be 4-D NCHW");
    const gc_shape p{x.size(0), x.size(1), cout, x.size(2), x.size(3), r, s, groups, sh, sw, ph, pw, dh, dw};
    int64_t ho = 0, wo = 0;
    int st = gc_validate_shape(&p, &ho, &wo);
    if (st != GC_OK) throw std::runtime_error("gc_status " + std::to_string(st) + ": " + gc_last_error());
    c10::OptionalDeviceGuard guard;
    if (x.is_cuda()) guard.reset_device(x.device());
    at::Tensor y = at::empty({p.n, cout, ho, wo}, x.options().memory_format(
                                                    layout == GC_B200_NHWC ? at::MemoryFormat::ChannelsLast
                                                                           : at::MemoryFormat::Contiguous));
    const gc_tensor xd = describe(x), wd = describe(w);
    gc_tensor yd = describe(y);
    gc_tensor bd{};
    if (bias.has_value()) bd = describe(*bias);
    void *stream = x.is_cuda() ? static_cast<void *>(c10::cuda::getCurrentCUDAStream(x.get_device()).stream())
                               : nullptr;
    st = gc_b200_conv_ex(&p, &xd, &wd, bias.has_value() ? &bd : nullptr, &yd, static_cast<int>(layout),
                         static_cast<int>(activation), stream);
    if (st != GC_OK) throw std::runtime_error("gc_status " + std::to_string(st) + ": " + gc_last_error());
    return y;
}

}  // namespace

PYBIND11_MODULE(_gcb_torch, m) {
    m.doc() = "gc_cuda_conv for torch tensors: output allocation and the C ABI call in C++";
    m.def("conv", &conv, "y = gc_cuda_conv(x, w) on the current CUDA stream");
    m.def("conv_ex", &conv_ex, "y = act(conv(x, w) + bias) through gc_b200_conv_ex on the current CUDA stream");
}
