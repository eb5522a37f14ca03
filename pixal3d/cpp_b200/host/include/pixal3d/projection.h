// Projection conditioning (image_attn_mode=proj producer), B200
// implementation.
//
// Same declarations as the reference's include/pixal3d/projection.h so
// callers compile unchanged.  The per-point projection and bilinear sampling
// run on the GPU (p3d_project_features in p3d.h): feature maps and
// coordinates are staged to device memory per call, the kernel computes in
// IEEE f32 in the reference's operation order, so the features and validity
// flags equal the reference's CPU results bit for bit.  Errors: return false
// and set *error when non-null, with the reference's messages.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace pixal3d {

struct SparseTensorF32;

// Camera of a projection view: horizontal FOV (radians), front-view
// distance, mesh scale, or a row-major camera-to-world matrix when
// has_transform is set.
struct ProjectionCamera {
    float camera_angle_x = 0.2f;
    float distance = 2.0f;
    float mesh_scale = 1.0f;
    bool has_transform = false;
    std::array<float, 16> transform_matrix{};

    static ProjectionCamera front(float camera_angle_x, float distance, float mesh_scale = 1.0f);
};

struct ProjectionGridOptions {
    int grid_resolution = 16;
    int image_resolution = 518;
};

// K x C features (K = grid_resolution^3, meshgrid "ij" point order) and one
// validity flag per point.
struct ProjectedGrid {
    int grid_resolution = 0;
    int channels = 0;
    std::vector<float> features;
    std::vector<std::uint8_t> valid;

    std::size_t points() const;
    bool empty() const;
};

// One H x W x C row-major f32 image feature map and its camera.
struct ProjectionView {
    const float *feature_map = nullptr;
    int height = 0;
    int width = 0;
    int channels = 0;
    ProjectionCamera camera;
};

// Every grid cell projected into the view and sampled with
// grid_sample(mode=bilinear, align_corners=False, padding_mode=border).
bool project_grid_features(const float *feature_map, int height, int width, int channels,
                           const ProjectionGridOptions &options, const ProjectionCamera &camera,
                           ProjectedGrid &output, std::string *error = nullptr);

// The same for sparse [batch=0, x, y, z] coordinates only, in caller order.
bool project_grid_features_at_coords(const float *feature_map, int height, int width, int channels,
                                     const ProjectionGridOptions &options, const ProjectionCamera &camera,
                                     const std::vector<std::int32_t> &coords, std::vector<float> &features,
                                     std::vector<std::uint8_t> &valid, std::string *error = nullptr);

// Mean over views of the dense projection; valid where any view is valid.
bool project_grid_features_average(const std::vector<ProjectionView> &views, const ProjectionGridOptions &options,
                                   ProjectedGrid &output, std::string *error = nullptr);

// Rows of a projected dense grid at sparse [0, x, y, z] coordinates.
bool projected_grid_to_sparse_f32(const ProjectedGrid &grid, const std::vector<std::int32_t> &coords,
                                  SparseTensorF32 &output, std::string *error = nullptr);

// relative[i] = F(distance[0]) * inverse(c2w[0]) * c2w[i].
bool compute_relative_calc_matrices(const std::vector<std::array<float, 16>> &camera_to_world,
                                    const std::vector<float> &distances,
                                    std::vector<std::array<float, 16>> &relative, std::string *error = nullptr);

}  // namespace pixal3d
