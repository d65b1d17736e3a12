// Minimal pybind module over the reference's voxelizer host functions, used only to build the
// reference into oracle/_ref/ as a test oracle (bit-exact CSR pin and the GPU comparator).
// The reference's own bindings.cpp also binds its feature-loss op, which the oracle does not need.
#include <torch/extension.h>

#include "cuda_gaussian_voxelizer.cuh"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    namespace gv = cudaprocess::gaussian_voxelizer;
    m.def("gaussian_voxelizer_forward", &gv::cuda_gaussian_voxelizer_forward, py::arg("means3D"),
          py::arg("opacity"), py::arg("covariances"), py::arg("voxel_size"), py::arg("voxel_range"),
          py::arg("features") = py::none());
    m.def("gaussian_voxelizer_backward", &gv::cuda_gaussian_voxelizer_backward, py::arg("grad_output"),
          py::arg("grad_feats_output"), py::arg("means3D"), py::arg("opacity"), py::arg("cov_inv"),
          py::arg("voxel_size"), py::arg("voxel_range"), py::arg("valid_voxel_lb"), py::arg("valid_voxel_ub"),
          py::arg("num_voxels_per_gaussian"), py::arg("g2t_offsets"), py::arg("g2t_tile_ids"),
          py::arg("density"), py::arg("grid_feats"), py::arg("features") = py::none());
}
