// Drives include/pixal3d/projection.h of the B200 library the way a caller
// of the reference does, on the inputs of the reference's projection fixture
// (a 5 x 4 x 3 map base + i/8 + (i % 7)/32; a front camera (0.8, 2.25, 1.5)
// and the same camera moved by x += 0.5; grid 4, image 16), and prints the
// results in the fixture's "name count values..." format so the test can
// compare them with the reference's own output.  Then checks the API's
// refusals, printing "error <message>" lines.
#include <array>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "pixal3d/projection.h"
#include "pixal3d/sparse.h"

namespace {

std::vector<float> fixture_map(float base) {
    std::vector<float> v(60);
    for (std::size_t i = 0; i < v.size(); ++i)
        v[i] = base + 0.125f * static_cast<float>(i) + 0.03125f * static_cast<float>(i % 7);
    return v;
}

void print(const char *name, const std::vector<float> &v) {
    std::printf("%s %zu", name, v.size());
    for (float x : v) std::printf(" %.9g", x);
    std::printf("\n");
}

void print(const char *name, const std::vector<std::uint8_t> &v) {
    std::printf("%s %zu", name, v.size());
    for (std::uint8_t x : v) std::printf(" %u", static_cast<unsigned>(x));
    std::printf("\n");
}

void report(bool ok, const std::string &err) { std::printf("error %s\n", ok ? "(none)" : err.c_str()); }

}  // namespace

int main() {
    using namespace pixal3d;
    ProjectionGridOptions options;
    options.grid_resolution = 4;
    options.image_resolution = 16;
    const std::vector<float> a = fixture_map(-0.5f), b = fixture_map(0.75f);
    const ProjectionCamera cam = ProjectionCamera::front(0.8f, 2.25f, 1.5f);
    std::string err;

    ProjectedGrid single;
    if (!project_grid_features(a.data(), 5, 4, 3, options, cam, single, &err)) {
        std::fprintf(stderr, "%s\n", err.c_str());
        return 1;
    }
    print("single_features", single.features);
    print("single_valid", single.valid);

    ProjectionCamera moved = cam;
    moved.has_transform = true;
    moved.transform_matrix = {{1, 0, 0, 0.5f, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1}};
    ProjectedGrid average;
    if (!project_grid_features_average({ProjectionView{a.data(), 5, 4, 3, cam}, ProjectionView{b.data(), 5, 4, 3, moved}},
                                       options, average, &err)) {
        std::fprintf(stderr, "%s\n", err.c_str());
        return 1;
    }
    print("average_features", average.features);
    print("average_valid", average.valid);

    const std::array<float, 16> eye = {{1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1}};
    std::vector<std::array<float, 16>> rel;
    if (!compute_relative_calc_matrices({eye, moved.transform_matrix}, {2.25f, 2.25f}, rel, &err)) {
        std::fprintf(stderr, "%s\n", err.c_str());
        return 1;
    }
    std::vector<float> flat;
    for (const auto &m : rel) flat.insert(flat.end(), m.begin(), m.end());
    print("relative_matrices", flat);

    // sparse rows in caller order (a repeated cell included) and the bridge
    std::vector<float> sf;
    std::vector<std::uint8_t> sv;
    const std::vector<std::int32_t> coords = {0, 3, 1, 2, 0, 0, 0, 0, 0, 3, 1, 2, 0, 2, 3, 1};
    if (!project_grid_features_at_coords(a.data(), 5, 4, 3, options, cam, coords, sf, sv, &err)) {
        std::fprintf(stderr, "%s\n", err.c_str());
        return 1;
    }
    print("sparse_features", sf);
    print("sparse_valid", sv);
    SparseTensorF32 bridged;
    report(projected_grid_to_sparse_f32(single, coords, bridged, &err), err);  // duplicate cell
    if (!projected_grid_to_sparse_f32(single, {0, 3, 1, 2, 0, 0, 0, 0, 0, 2, 3, 1}, bridged, &err)) {
        std::fprintf(stderr, "%s\n", err.c_str());
        return 1;
    }
    print("bridge_features", bridged.feats);

    // refusals
    ProjectionGridOptions bad = options;
    bad.grid_resolution = 0;
    ProjectedGrid g;
    report(project_grid_features(a.data(), 5, 4, 3, bad, cam, g, &err), err);
    report(project_grid_features(a.data(), 5, 4, 3, options, ProjectionCamera::front(3.5f, 2.0f), g, &err), err);
    ProjectionCamera singular = cam;
    singular.has_transform = true;
    singular.transform_matrix = {};
    report(project_grid_features(a.data(), 5, 4, 3, options, singular, g, &err), err);
    report(project_grid_features(nullptr, 5, 4, 3, options, cam, g, &err), err);
    report(project_grid_features_average({}, options, g, &err), err);
    report(project_grid_features_average({ProjectionView{a.data(), 5, 4, 3, cam}, ProjectionView{a.data(), 5, 6, 2, cam}},
                                         options, g, &err),
           err);
    report(project_grid_features_at_coords(a.data(), 5, 4, 3, options, cam, {0, 1, 1}, sf, sv, &err), err);
    report(project_grid_features_at_coords(a.data(), 5, 4, 3, options, cam, {1, 0, 0, 0}, sf, sv, &err), err);
    report(project_grid_features_at_coords(a.data(), 5, 4, 3, options, cam, {0, 0, 4, 0}, sf, sv, &err), err);
    report(projected_grid_to_sparse_f32(single, {0, 0, 0, 9}, bridged, &err), err);
    report(compute_relative_calc_matrices({eye}, {2.0f, 1.0f}, rel, &err), err);
    report(compute_relative_calc_matrices({std::array<float, 16>{}}, {2.0f}, rel, &err), err);
    return 0;
}
