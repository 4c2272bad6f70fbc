// Python binding of the reference's NerfMlp for the GPU checks (TEST INFRASTRUCTURE ONLY): the reference class
// (mlp/include/nerf_mlp.h:34-73, mlp/src/nerf_mlp.cu) compiled from where it lies, exposed under the names its own
// module uses (torch_bindings/bindings.cu:23-30), so that a test can run the reference's cuBLASLt chain beside this
// backend's tensor-core kernels on the same tensors.
#include <torch/extension.h>

#include "nerf_mlp.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("nerf_mlp_parameters", &zipnerf::mlp::nerf_mlp_parameters);
    py::class_<zipnerf::mlp::NerfMlp>(m, "NerfMlp")
        .def(py::init<int64_t, int64_t, int64_t, int64_t, int64_t>())
        .def_property_readonly("n_features", &zipnerf::mlp::NerfMlp::n_features)
        .def_property_readonly("n_inputs", &zipnerf::mlp::NerfMlp::n_inputs)
        .def("pack", &zipnerf::mlp::NerfMlp::pack)
        .def("forward", &zipnerf::mlp::NerfMlp::forward)
        .def("backward", &zipnerf::mlp::NerfMlp::backward);
}
