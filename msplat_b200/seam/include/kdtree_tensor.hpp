// kdtree_tensor.hpp for the CUDA seam build: the reference's PointsTensor
// (core/include/kdtree_tensor.hpp, a nanoflann k-d tree searched on the
// host) with the same interface, its k-nearest-neighbour search run on the
// GPU by the engine (msplat_knn_mean_distance: an exact grid search, so the
// same k smallest squared distances, formed as nanoflann's L2_Simple_Adaptor
// forms them).  Model::Model (model.cpp:65-75) uses scales(4) for the
// initial Gaussian sizes.
#ifndef KDTREE_TENSOR_H
#define KDTREE_TENSOR_H

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "seam_engine.h"

struct PointsTensor {
    const float* data;
    int64_t count;

    PointsTensor(const float* data, int64_t count) : data(data), count(count) {}

    // Mean distance to the k-1 nearest other points, per point.
    std::vector<float> scales(int k = 4) const
    {
        std::vector<float> result((size_t)count);
        if (count > 0 && seam::knn_mean_distance(data, count, k, result.data()) != 0)
            throw std::runtime_error(std::string("PointsTensor::scales: ") + seam::last_error());
        return result;
    }
};

#endif
