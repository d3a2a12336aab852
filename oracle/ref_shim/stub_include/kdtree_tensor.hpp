// kdtree_tensor.hpp stand-in for building the reference's model.cpp without
// nanoflann (its CMake fetches nanoflann v1.5.5 at configure time; there is
// no copy here).  Same interface as core/include/kdtree_tensor.hpp:
// PointsTensor(data, count).scales(k) = mean distance to the k-1 nearest
// other points.  The k-d tree search is exact, so an exhaustive search finds
// the same k smallest squared distances, formed as nanoflann's
// L2_Simple_Adaptor forms them (result += diff * diff over x, y, z).
//
// TEST INFRASTRUCTURE ONLY (oracle/ref_shim/build_ref.py build_trainer).
#ifndef KDTREE_TENSOR_H
#define KDTREE_TENSOR_H

#include <cfloat>
#include <cmath>
#include <cstdint>
#include <vector>

struct PointsTensor {
    const float* data;
    int64_t count;

    PointsTensor(const float* d, int64_t n) : data(d), count(n) {}

    std::vector<float> scales(int k = 4) const
    {
        std::vector<float> result(count);
#pragma omp parallel for schedule(dynamic, 256)
        for (int64_t i = 0; i < count; i++) {
            std::vector<float> best(k, FLT_MAX);
            const float* q = &data[i * 3];
            for (int64_t j = 0; j < count; j++) {
                float d = 0.0f;
                for (int a = 0; a < 3; a++) {
                    const float diff = q[a] - data[j * 3 + a];
                    d += diff * diff;
                }
                if (d < best[k - 1]) {
                    int m = k - 1;
                    while (m > 0 && best[m - 1] > d) {
                        best[m] = best[m - 1];
                        m--;
                    }
                    best[m] = d;
                }
            }
            float sum = 0;
            for (int j = 1; j < k; j++) sum += std::sqrt(best[j]);
            result[i] = sum / (k - 1);
        }
        return result;
    }
};

#endif
