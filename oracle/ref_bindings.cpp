// Minimal pybind module over the reference's voxelizer and feature-loss host functions, used only to
// build the reference into oracle/_ref/ as a test oracle (bit-exact CSR pin and the GPU comparator).
// The names and argument lists are those of the reference's own src/bindings.cpp:8-100.
#include <torch/extension.h>

#include "cuda_feats_loss.cuh"
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
    namespace fl = cudaprocess::feats_loss;
    m.def("CudaFeatsCosinelossForward", &fl::CudaFeatsCosinelossForward, py::arg("voxel_label"),
          py::arg("occ_gt_mask_camera"), py::arg("d_grid_feats"), py::arg("pseudo_dino_gt"));
    m.def("CudaFeatsCosinelossBackward", &fl::CudaFeatsCosinelossBackward, py::arg("grad_output"),
          py::arg("voxel_label"), py::arg("occ_gt_mask_camera"), py::arg("d_grid_feats"),
          py::arg("pseudo_dino_gt"), py::arg("num_valid_voxel"));
}
