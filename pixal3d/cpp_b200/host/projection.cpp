// include/pixal3d/projection.h on the B200 kernels: each call stages the
// feature maps (and coordinates) to device memory, runs
// p3d_project_features and copies features and flags back.
#include "pixal3d/projection.h"

#include <algorithm>
#include <cmath>

#include "device.h"
#include "pixal3d/sparse.h"

namespace pixal3d {

using b200::Buffer;
using b200::fail;
using b200::ok;

namespace {

p3d_projection_view to_view(const float *dev_map, int height, int width, int channels, int image_resolution,
                            const ProjectionCamera &camera) {
    p3d_projection_view v{};
    v.feature_map = dev_map;
    v.height = height;
    v.width = width;
    v.channels = channels;
    v.image_resolution = image_resolution;
    v.camera_angle_x = camera.camera_angle_x;
    v.distance = camera.distance;
    v.mesh_scale = camera.mesh_scale;
    v.has_transform = camera.has_transform ? 1 : 0;
    for (int i = 0; i < 16; ++i) v.transform_matrix[i] = camera.transform_matrix[static_cast<std::size_t>(i)];
    return v;
}

// Host views -> device maps + p3d views.  Maps are uploaded only after the
// shape checks, which p3d_project_features repeats with the same messages.
bool stage_views(p3d_ctx *ctx, const std::vector<ProjectionView> &views, int image_resolution,
                 std::vector<Buffer> &maps, std::vector<p3d_projection_view> &out, std::string *error) {
    maps.resize(views.size());
    out.resize(views.size());
    for (std::size_t i = 0; i < views.size(); ++i) {
        const ProjectionView &v = views[i];
        const float *dev = nullptr;
        if (v.feature_map && v.height > 0 && v.width > 0 && v.channels > 0) {
            const std::size_t bytes = sizeof(float) * static_cast<std::size_t>(v.height) * v.width * v.channels;
            if (!b200::upload(ctx, maps[i], v.feature_map, bytes, error)) return false;
            dev = maps[i].as<float>();
        }
        out[i] = to_view(dev, v.height, v.width, v.channels, image_resolution, v.camera);
        if (!v.feature_map) out[i].feature_map = nullptr;
    }
    return true;
}

bool run_projection(const std::vector<ProjectionView> &views, const ProjectionGridOptions &options,
                    const std::vector<std::int32_t> *coords, std::vector<float> &features,
                    std::vector<std::uint8_t> &valid, std::string *error) {
    p3d_ctx *ctx = b200::context(error);
    if (!ctx) return false;
    std::vector<Buffer> maps;
    std::vector<p3d_projection_view> pv;
    if (!stage_views(ctx, views, options.image_resolution, maps, pv, error)) return false;
    const int r = options.grid_resolution;
    const int64_t n = coords ? static_cast<int64_t>(coords->size() / 4)
                             : (r > 0 ? static_cast<int64_t>(r) * r * r : 0);
    const int channels = views.empty() ? 0 : views.front().channels;
    Buffer dc, out, dv;
    if (coords && !coords->empty() && !b200::upload(ctx, dc, coords->data(), coords->size() * 4, error)) return false;
    if (n > 0 && channels > 0 &&
        (!out.allocate(ctx, sizeof(float) * static_cast<std::size_t>(n) * channels, error) ||
         !dv.allocate(ctx, static_cast<std::size_t>(n), error)))
        return false;
    // An empty sparse list (n == 0) still goes through the option and camera checks.
    if (!ok(ctx,
            p3d_project_features(ctx, pv.data(), static_cast<int>(pv.size()), r, dc.as<int32_t>(), n, out.get(),
                                 channels, P3D_F32, dv.as<uint8_t>()),
            error))
        return false;
    features.resize(static_cast<std::size_t>(n) * static_cast<std::size_t>(channels));
    valid.resize(static_cast<std::size_t>(n));
    if (n == 0) return true;
    return b200::download(ctx, features.data(), out, features.size() * sizeof(float), error) &&
           b200::download(ctx, valid.data(), dv, valid.size(), error);
}

}  // namespace

ProjectionCamera ProjectionCamera::front(float camera_angle_x, float distance, float mesh_scale) {
    ProjectionCamera camera;
    camera.camera_angle_x = camera_angle_x;
    camera.distance = distance;
    camera.mesh_scale = mesh_scale;
    camera.has_transform = false;
    return camera;
}

std::size_t ProjectedGrid::points() const {
    const std::size_t r = grid_resolution > 0 ? static_cast<std::size_t>(grid_resolution) : 0;
    return r * r * r;
}

bool ProjectedGrid::empty() const { return features.empty(); }

bool project_grid_features(const float *feature_map, int height, int width, int channels,
                           const ProjectionGridOptions &options, const ProjectionCamera &camera,
                           ProjectedGrid &output, std::string *error) {
    ProjectionView view{feature_map, height, width, channels, camera};
    return project_grid_features_average({view}, options, output, error);
}

bool project_grid_features_at_coords(const float *feature_map, int height, int width, int channels,
                                     const ProjectionGridOptions &options, const ProjectionCamera &camera,
                                     const std::vector<std::int32_t> &coords, std::vector<float> &features,
                                     std::vector<std::uint8_t> &valid, std::string *error) {
    features.clear();
    valid.clear();
    if (coords.size() % 4 != 0) {
        // the option / camera checks come first, as in the reference
        std::vector<std::int32_t> none;
        std::vector<float> f;
        std::vector<std::uint8_t> v;
        ProjectionView view{feature_map, height, width, channels, camera};
        if (!run_projection({view}, options, &none, f, v, error)) return false;
        return fail(error, "sparse projection coordinates must contain [batch,x,y,z] rows");
    }
    const int r = options.grid_resolution;
    for (std::size_t i = 0; i < coords.size(); i += 4) {
        if (coords[i] != 0 || coords[i + 1] < 0 || coords[i + 2] < 0 || coords[i + 3] < 0 || coords[i + 1] >= r ||
            coords[i + 2] >= r || coords[i + 3] >= r) {
            // report option errors first (the reference validates them before the loop)
            std::vector<std::int32_t> none;
            std::vector<float> f;
            std::vector<std::uint8_t> v;
            ProjectionView view{feature_map, height, width, channels, camera};
            if (!run_projection({view}, options, &none, f, v, error)) return false;
            return fail(error, "sparse projection coordinate is outside the requested grid");
        }
    }
    ProjectionView view{feature_map, height, width, channels, camera};
    if (!run_projection({view}, options, &coords, features, valid, error)) {
        features.clear();
        valid.clear();
        return false;
    }
    return true;
}

bool project_grid_features_average(const std::vector<ProjectionView> &views, const ProjectionGridOptions &options,
                                   ProjectedGrid &output, std::string *error) {
    if (views.empty()) return fail(error, "at least one projection view is required");
    std::vector<float> features;
    std::vector<std::uint8_t> valid;
    if (!run_projection(views, options, nullptr, features, valid, error)) return false;
    output.grid_resolution = options.grid_resolution;
    output.channels = views.front().channels;
    output.features = std::move(features);
    output.valid = std::move(valid);
    return true;
}

bool projected_grid_to_sparse_f32(const ProjectedGrid &grid, const std::vector<std::int32_t> &coords,
                                  SparseTensorF32 &output, std::string *error) {
    output = SparseTensorF32{};
    if (grid.grid_resolution <= 0 || grid.channels <= 0 ||
        grid.features.size() != grid.points() * static_cast<std::size_t>(grid.channels) || coords.size() % 4 != 0)
        return fail(error, "invalid projected grid or sparse coordinate list");
    // A row copy between host buffers (no arithmetic): the grid and the
    // result are host vectors in this API.
    const int r = grid.grid_resolution;
    const std::size_t c = static_cast<std::size_t>(grid.channels);
    const std::size_t n = coords.size() / 4;
    output.batch_size = 1;
    output.channels = grid.channels;
    output.spatial_x = output.spatial_y = output.spatial_z = r;
    output.coords = coords;
    output.feats.resize(n * c);
    for (std::size_t p = 0; p < n; ++p) {
        const std::int32_t b = coords[4 * p], x = coords[4 * p + 1], y = coords[4 * p + 2], z = coords[4 * p + 3];
        if (b != 0 || x < 0 || x >= r || y < 0 || y >= r || z < 0 || z >= r) {
            output = SparseTensorF32{};
            return fail(error, "projected sparse coordinate is outside the dense grid");
        }
        const std::size_t g = (static_cast<std::size_t>(x) * r + static_cast<std::size_t>(y)) * r +
                              static_cast<std::size_t>(z);
        std::copy(grid.features.begin() + static_cast<std::ptrdiff_t>(g * c),
                  grid.features.begin() + static_cast<std::ptrdiff_t>((g + 1) * c),
                  output.feats.begin() + static_cast<std::ptrdiff_t>(p * c));
    }
    return output.valid(error);
}

bool compute_relative_calc_matrices(const std::vector<std::array<float, 16>> &camera_to_world,
                                    const std::vector<float> &distances,
                                    std::vector<std::array<float, 16>> &relative, std::string *error) {
    if (camera_to_world.empty()) return fail(error, "at least one camera transform is required");
    if (camera_to_world.size() != distances.size())
        return fail(error, "camera transform and distance counts must match");
    if (!(distances[0] > 0.0f) || !std::isfinite(distances[0]))
        return fail(error, "main-view distance must be finite and positive");
    std::vector<float> flat(camera_to_world.size() * 16), out(flat.size());
    for (std::size_t i = 0; i < camera_to_world.size(); ++i)
        std::copy(camera_to_world[i].begin(), camera_to_world[i].end(), flat.begin() + static_cast<std::ptrdiff_t>(16 * i));
    if (p3d_projection_relative_matrices(nullptr, flat.data(), distances.data(),
                                         static_cast<int>(camera_to_world.size()), out.data()) != P3D_OK)
        return fail(error, "main-view camera transform matrix is singular");
    relative.resize(camera_to_world.size());
    for (std::size_t i = 0; i < relative.size(); ++i)
        std::copy(out.begin() + static_cast<std::ptrdiff_t>(16 * i), out.begin() + static_cast<std::ptrdiff_t>(16 * i + 16),
                  relative[i].begin());
    return true;
}

}  // namespace pixal3d
