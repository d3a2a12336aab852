// io.cu -- checkpoint (.msplat), PLY and .splat files of a Gaussian model.
//
// Host code over the engine's device buffers: the training step keeps
// parameters on the GPU, so a save copies them to the host (after the
// engine's stream has drained, as the reference's msplat_gpu_sync does) and
// a load copies them back.  Every array argument may also be host memory
// (pointers the CUDA runtime does not know are read and written directly),
// which lets the formats be checked without a GPU.
//
// Formats, byte for byte those of the reference:
//   .msplat  Model::saveCheckpoint / loadCheckpoint (core/src/model.cpp:333-488)
//   .ply     saveGaussianPly / loadGaussianPly (core/src/loaders/save_gaussians.cpp:10-55,
//            104-190)
//   .splat   saveGaussianSplat (save_gaussians.cpp:57-102)
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <numeric>
#include <string>
#include <vector>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

constexpr uint32_t kCkptMagic = 0x4C50534D;  // "MSPL"
constexpr uint32_t kCkptVersion = 1;
constexpr int kWidths[kGroups - 1] = {3, 3, 4, 3};  // means, scales, quats, dc (rest, opacity apart)

bool is_device(const void* p)
{
    if (!p) return false;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();  // no device, or an unknown pointer: host memory
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

// Waits for the engine's queued work once a device buffer is involved.
void drain_engine()
{
    std::lock_guard<std::mutex> lk(engine_mutex());
    if (engine_init() == MSPLAT_OK) cudaStreamSynchronize(engine_stream());
}

int fetch(const float* src, size_t n, std::vector<float>& out)
{
    out.resize(n);
    if (n == 0) return MSPLAT_OK;
    if (is_device(src)) {
        if (cudaMemcpy(out.data(), src, n * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess) {
            set_error("device-to-host copy of %zu floats failed", n);
            return MSPLAT_ERR_CUDA;
        }
    } else {
        std::memcpy(out.data(), src, n * sizeof(float));
    }
    return MSPLAT_OK;
}

int store(float* dst, const float* src, size_t n)
{
    if (n == 0) return MSPLAT_OK;
    if (is_device(dst)) {
        if (cudaMemcpy(dst, src, n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
            set_error("host-to-device copy of %zu floats failed", n);
            return MSPLAT_ERR_CUDA;
        }
    } else {
        std::memcpy(dst, src, n * sizeof(float));
    }
    return MSPLAT_OK;
}

bool any_device(const float* const* ps, int n)
{
    for (int i = 0; i < n; i++)
        if (is_device(ps[i])) return true;
    return false;
}

// Shapes of the six groups (group order means, scales, quats, dc, rest, opacity).
std::vector<int64_t> group_shape(int g, int64_t n, int rest_bases)
{
    switch (g) {
        case 4: return {n, rest_bases, 3};
        case 5: return {n, 1};
        default: return {n, kWidths[g]};
    }
}

size_t group_width(int g, int rest_bases) { return g == 4 ? 3 * (size_t)rest_bases : g == 5 ? 1 : kWidths[g]; }

template <class T>
void put(std::ofstream& f, const T& v) { f.write(reinterpret_cast<const char*>(&v), sizeof(T)); }
template <class T>
bool get(std::ifstream& f, T& v) { return (bool)f.read(reinterpret_cast<char*>(&v), sizeof(T)); }

// writeTensor (model.cpp:340-350): ndim, shape, byte count, raw data
void write_tensor(std::ofstream& f, const std::vector<int64_t>& shape, const std::vector<float>& data)
{
    put(f, (uint32_t)shape.size());
    for (int64_t s : shape) put(f, s);
    put(f, (uint64_t)(data.size() * sizeof(float)));
    f.write(reinterpret_cast<const char*>(data.data()), data.size() * sizeof(float));
}

// readTensor (model.cpp:352-363); checks the shape against what is expected
int read_tensor(std::ifstream& f, const std::vector<int64_t>& want, std::vector<float>& out)
{
    uint32_t ndim = 0;
    if (!get(f, ndim) || ndim != want.size()) {
        set_error("checkpoint: tensor of %u dimensions where %zu are expected", ndim, want.size());
        return MSPLAT_ERR_ARG;
    }
    size_t numel = 1;
    for (uint32_t i = 0; i < ndim; i++) {
        int64_t s = 0;
        if (!get(f, s) || s != want[i]) {
            set_error("checkpoint: tensor shape does not match its header");
            return MSPLAT_ERR_ARG;
        }
        numel *= (size_t)s;
    }
    uint64_t bytes = 0;
    if (!get(f, bytes) || bytes != numel * sizeof(float)) {
        set_error("checkpoint: tensor byte count does not match its shape");
        return MSPLAT_ERR_ARG;
    }
    out.resize(numel);
    if (!f.read(reinterpret_cast<char*>(out.data()), (std::streamsize)bytes)) {
        set_error("checkpoint: file ends inside a tensor");
        return MSPLAT_ERR_ARG;
    }
    return MSPLAT_OK;
}

struct CkptHeader {
    uint32_t step, num, sh_degree, adam_steps;
    float lr[kGroups], lr_init, lr_final;
    int rest_bases;
};

// Header and scalar state (model.cpp:365-382, 404-422), plus the SH-rest
// basis count read from the features_rest tensor's shape.
int read_header(std::ifstream& f, const char* path, CkptHeader& h)
{
    uint32_t magic = 0, version = 0;
    if (!get(f, magic) || magic != kCkptMagic) {
        set_error("%s: not a valid msplat checkpoint file", path);
        return MSPLAT_ERR_ARG;
    }
    if (!get(f, version) || version != kCkptVersion) {
        set_error("%s: unsupported checkpoint version %u", path, version);
        return MSPLAT_ERR_ARG;
    }
    bool ok = get(f, h.step) && get(f, h.num) && get(f, h.sh_degree) && get(f, h.adam_steps);
    for (int g = 0; g < kGroups; g++) ok = ok && get(f, h.lr[g]);
    ok = ok && get(f, h.lr_init) && get(f, h.lr_final);
    if (!ok) {
        set_error("%s: checkpoint header is truncated", path);
        return MSPLAT_ERR_ARG;
    }
    // the features_rest tensor comes after means, scales, quats and dc
    const std::streampos data_start = f.tellg();
    for (int g = 0; g < 4; g++) {
        uint32_t ndim = 0;
        if (!get(f, ndim) || ndim > 8) {
            set_error("%s: checkpoint tensor %d is malformed", path, g);
            return MSPLAT_ERR_ARG;
        }
        f.seekg(8 * (std::streamoff)ndim, std::ios::cur);
        uint64_t bytes = 0;
        if (!get(f, bytes)) {
            set_error("%s: checkpoint is truncated", path);
            return MSPLAT_ERR_ARG;
        }
        f.seekg((std::streamoff)bytes, std::ios::cur);
    }
    uint32_t ndim = 0;
    int64_t shape[3] = {0, 0, 0};
    if (!get(f, ndim) || ndim != 3 || !get(f, shape[0]) || !get(f, shape[1]) || !get(f, shape[2]) ||
        shape[2] != 3) {
        set_error("%s: checkpoint has no [N, bases, 3] features_rest tensor", path);
        return MSPLAT_ERR_ARG;
    }
    h.rest_bases = (int)shape[1];
    f.seekg(data_start);
    return MSPLAT_OK;
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_save_checkpoint(const char* path, int step, int num_active, int sh_degree,
                           int adam_step_count, const float* adam_lr, float means_lr_init,
                           float means_lr_final, int features_rest_bases,
                           const float* const* params, const float* const* exp_avg,
                           const float* const* exp_avg_sq)
{
    if (!path || num_active < 0 || features_rest_bases < 0 || !adam_lr || !params || !exp_avg ||
        !exp_avg_sq) {
        set_error("msplat_save_checkpoint: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    if (any_device(params, kGroups) || any_device(exp_avg, kGroups) ||
        any_device(exp_avg_sq, kGroups))
        drain_engine();
    std::ofstream f(path, std::ios::binary);
    if (!f.is_open()) {
        set_error("cannot open checkpoint file for writing: %s", path);
        return MSPLAT_ERR_ARG;
    }
    put(f, kCkptMagic);
    put(f, kCkptVersion);
    put(f, (uint32_t)step);
    put(f, (uint32_t)num_active);
    put(f, (uint32_t)sh_degree);
    put(f, (uint32_t)adam_step_count);
    for (int g = 0; g < kGroups; g++) put(f, adam_lr[g]);
    put(f, means_lr_init);
    put(f, means_lr_final);
    std::vector<float> buf;
    const float* const* sets[3] = {params, exp_avg, exp_avg_sq};
    for (int s = 0; s < 3; s++)
        for (int g = 0; g < kGroups; g++) {
            int rc = fetch(sets[s][g], (size_t)num_active * group_width(g, features_rest_bases), buf);
            if (rc) return rc;
            write_tensor(f, group_shape(g, num_active, features_rest_bases), buf);
        }
    if (!f.good()) {
        set_error("writing checkpoint %s failed", path);
        return MSPLAT_ERR_ARG;
    }
    return MSPLAT_OK;
}

int msplat_read_checkpoint_header(const char* path, int* step, int* num_active, int* sh_degree,
                                  int* adam_step_count, float* adam_lr, float* means_lr_init,
                                  float* means_lr_final, int* features_rest_bases)
{
    if (!path) {
        set_error("msplat_read_checkpoint_header: null path");
        return MSPLAT_ERR_ARG;
    }
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) {
        set_error("cannot open checkpoint file: %s", path);
        return MSPLAT_ERR_ARG;
    }
    CkptHeader h{};
    int rc = read_header(f, path, h);
    if (rc) return rc;
    if (step) *step = (int)h.step;
    if (num_active) *num_active = (int)h.num;
    if (sh_degree) *sh_degree = (int)h.sh_degree;
    if (adam_step_count) *adam_step_count = (int)h.adam_steps;
    if (adam_lr) std::memcpy(adam_lr, h.lr, sizeof(h.lr));
    if (means_lr_init) *means_lr_init = h.lr_init;
    if (means_lr_final) *means_lr_final = h.lr_final;
    if (features_rest_bases) *features_rest_bases = h.rest_bases;
    return MSPLAT_OK;
}

int msplat_load_checkpoint(const char* path, int capacity, float* const* params,
                           float* const* exp_avg, float* const* exp_avg_sq)
{
    if (!path || !params || !exp_avg || !exp_avg_sq) {
        set_error("msplat_load_checkpoint: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) {
        set_error("cannot open checkpoint file: %s", path);
        return MSPLAT_ERR_ARG;
    }
    CkptHeader h{};
    int rc = read_header(f, path, h);
    if (rc) return rc;
    if ((long long)h.num > capacity) {
        set_error("checkpoint %s holds %u Gaussians, more than the %d rows given", path, h.num,
                  capacity);
        return MSPLAT_ERR_ARG;
    }
    std::vector<float> buf;
    float* const* sets[3] = {params, exp_avg, exp_avg_sq};
    for (int s = 0; s < 3; s++)
        for (int g = 0; g < kGroups; g++) {
            if ((rc = read_tensor(f, group_shape(g, h.num, h.rest_bases), buf))) return rc;
            if ((rc = store(sets[s][g], buf.data(), buf.size()))) return rc;
        }
    return (int)h.step;
}

// saveGaussianPly (save_gaussians.cpp:10-55)
int msplat_save_ply(const char* path, int step, int n, int features_rest_bases,
                    const float* const* params, int keep_crs, float scale,
                    const float* translation)
{
    if (!path || n < 0 || features_rest_bases < 0 || !params || (keep_crs && !translation)) {
        set_error("msplat_save_ply: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    if (any_device(params, kGroups)) drain_engine();
    std::vector<float> g[kGroups];
    for (int i = 0; i < kGroups; i++) {
        int rc = fetch(params[i], (size_t)n * group_width(i, features_rest_bases), g[i]);
        if (rc) return rc;
    }
    std::ofstream o(path, std::ios::binary);
    if (!o.is_open()) {
        set_error("cannot open PLY file for writing: %s", path);
        return MSPLAT_ERR_ARG;
    }
    const int num_dc = 3, fr_bases = features_rest_bases, num_fr = 3 * fr_bases;
    o << "ply\nformat binary_little_endian 1.0\n";
    o << "comment msplat v" << step << "\n";
    o << "element vertex " << (int64_t)n << "\n";
    o << "property float x\nproperty float y\nproperty float z\n";
    o << "property float nx\nproperty float ny\nproperty float nz\n";
    for (int i = 0; i < num_dc; i++) o << "property float f_dc_" << i << "\n";
    for (int i = 0; i < num_fr; i++) o << "property float f_rest_" << i << "\n";
    o << "property float opacity\n";
    o << "property float scale_0\nproperty float scale_1\nproperty float scale_2\n";
    o << "property float rot_0\nproperty float rot_1\nproperty float rot_2\nproperty float rot_3\n";
    o << "end_header\n";
    const int per_row = 3 + 3 + num_dc + num_fr + 1 + 3 + 4;
    std::vector<float> row(per_row);
    for (int64_t i = 0; i < n; i++) {
        int c = 0;
        for (int j = 0; j < 3; j++)
            row[c++] = keep_crs ? (g[0][i * 3 + j] / scale + translation[j]) : g[0][i * 3 + j];
        row[c++] = 0;
        row[c++] = 0;
        row[c++] = 0;
        for (int j = 0; j < num_dc; j++) row[c++] = g[3][i * num_dc + j];
        // [bases, 3] -> [3, bases], the PLY convention
        for (int ch = 0; ch < 3; ch++)
            for (int b = 0; b < fr_bases; b++) row[c++] = g[4][i * fr_bases * 3 + b * 3 + ch];
        row[c++] = g[5][i];
        for (int j = 0; j < 3; j++)
            row[c++] = keep_crs ? std::log(std::exp(g[1][i * 3 + j]) / scale) : g[1][i * 3 + j];
        for (int j = 0; j < 4; j++) row[c++] = g[2][i * 4 + j];
        o.write(reinterpret_cast<const char*>(row.data()), per_row * sizeof(float));
    }
    if (!o.good()) {
        set_error("writing PLY %s failed", path);
        return MSPLAT_ERR_ARG;
    }
    return MSPLAT_OK;
}

// saveGaussianSplat (save_gaussians.cpp:57-102): 32-byte records sorted by
// size x opacity, largest first
int msplat_save_splat(const char* path, int n, const float* const* params, int keep_crs,
                      float scale, const float* translation)
{
    if (!path || n < 0 || !params || (keep_crs && !translation)) {
        set_error("msplat_save_splat: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    const int want[kGroups] = {0, 1, 2, 3, -1, 5};
    if (is_device(params[0]) || is_device(params[1]) || is_device(params[2]) ||
        is_device(params[3]) || is_device(params[5]))
        drain_engine();
    std::vector<float> g[kGroups];
    for (int i = 0; i < kGroups; i++) {
        if (want[i] < 0) continue;
        int rc = fetch(params[i], (size_t)n * group_width(i, 0), g[i]);
        if (rc) return rc;
    }
    std::ofstream o(path, std::ios::binary);
    if (!o.is_open()) {
        set_error("cannot open .splat file for writing: %s", path);
        return MSPLAT_ERR_ARG;
    }
    const double kC0 = 0.28209479177387814;
    std::vector<float> order(n);
    for (int64_t i = 0; i < n; i++) {
        float s = std::exp(g[1][i * 3]) + std::exp(g[1][i * 3 + 1]) + std::exp(g[1][i * 3 + 2]);
        if (keep_crs) s /= scale;
        order[i] = s / (1.0f + std::exp(-g[5][i]));
    }
    std::vector<size_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0);
    std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return order[a] > order[b]; });
    for (int64_t ii = 0; ii < n; ii++) {
        const size_t i = idx[ii];
        float m[3], sc[3];
        for (int j = 0; j < 3; j++)
            m[j] = keep_crs ? (g[0][i * 3 + j] / scale + translation[j]) : g[0][i * 3 + j];
        o.write(reinterpret_cast<const char*>(m), 12);
        for (int j = 0; j < 3; j++)
            sc[j] = keep_crs ? (std::exp(g[1][i * 3 + j]) / scale) : std::exp(g[1][i * 3 + j]);
        o.write(reinterpret_cast<const char*>(sc), 12);
        uint8_t rgb[3];
        for (int j = 0; j < 3; j++)
            rgb[j] = (uint8_t)std::clamp(((double)g[3][i * 3 + j] * kC0 + 0.5) * 255.0, 0.0, 255.0);
        o.write(reinterpret_cast<const char*>(rgb), 3);
        const float sig = 1.0f / (1.0f + std::exp(-g[5][i]));
        const uint8_t a = (uint8_t)std::clamp(sig * 255.0f, 0.0f, 255.0f);
        o.write(reinterpret_cast<const char*>(&a), 1);
        uint8_t q[4];
        for (int j = 0; j < 4; j++) q[j] = (uint8_t)std::clamp(g[2][i * 4 + j] * 128.0f + 128.0f, 0.0f, 255.0f);
        o.write(reinterpret_cast<const char*>(q), 4);
    }
    if (!o.good()) {
        set_error("writing .splat %s failed", path);
        return MSPLAT_ERR_ARG;
    }
    return MSPLAT_OK;
}

// The header part of loadGaussianPly (save_gaussians.cpp:104-135)
int msplat_read_ply_header(const char* path, int* n, int* step, int* features_rest_bases)
{
    std::ifstream f(path ? path : "", std::ios::binary);
    if (!path || !f.is_open()) {
        set_error("cannot open PLY file: %s", path ? path : "(null)");
        return MSPLAT_ERR_ARG;
    }
    std::string line;
    std::getline(f, line);
    if (line.find("ply") == std::string::npos) {
        set_error("not a PLY file: %s", path);
        return MSPLAT_ERR_ARG;
    }
    std::getline(f, line);
    int num = 0, st = 0, num_dc = 0, num_fr = 0;
    bool ended = false;
    while (std::getline(f, line)) {
        if (line == "end_header") {
            ended = true;
            break;
        }
        const std::string iter_prefix = "comment Generated by msplat at iteration ";
        if (line.rfind(iter_prefix, 0) == 0) st = std::atoi(line.c_str() + iter_prefix.size());
        const std::string vertex_prefix = "element vertex ";
        if (line.rfind(vertex_prefix, 0) == 0) num = std::atoi(line.c_str() + vertex_prefix.size());
        if (line.rfind("property float f_dc_", 0) == 0) num_dc++;
        if (line.rfind("property float f_rest_", 0) == 0) num_fr++;
    }
    if (!ended || num <= 0) {
        set_error("PLY %s has no vertices", path);
        return MSPLAT_ERR_ARG;
    }
    if (num_dc != 3 || num_fr % 3) {
        set_error("PLY %s: %d f_dc and %d f_rest properties (3 and a multiple of 3 expected)", path,
                  num_dc, num_fr);
        return MSPLAT_ERR_ARG;
    }
    if (n) *n = num;
    if (step) *step = st;
    if (features_rest_bases) *features_rest_bases = num_fr / 3;
    return MSPLAT_OK;
}

// loadGaussianPly (save_gaussians.cpp:104-190) into arrays of >= capacity rows
int msplat_load_ply(const char* path, int capacity, float* const* params, int keep_crs,
                    float scale, const float* translation)
{
    int n = 0, st = 0, fr_bases = 0;
    int rc = msplat_read_ply_header(path, &n, &st, &fr_bases);
    if (rc) return rc;
    if (!params || (keep_crs && !translation) || n > capacity) {
        set_error("msplat_load_ply: invalid arguments (%d vertices, %d rows given)", n, capacity);
        return MSPLAT_ERR_ARG;
    }
    std::ifstream f(path, std::ios::binary);
    std::string line;
    while (std::getline(f, line) && line != "end_header") {}
    const int num_fr = 3 * fr_bases;
    std::vector<float> means(3 * (size_t)n), dc(3 * (size_t)n), fr((size_t)n * num_fr), op(n),
        sc(3 * (size_t)n), qt(4 * (size_t)n), rest((size_t)n * num_fr);
    float normals[3];
    for (int i = 0; i < n; i++) {
        f.read(reinterpret_cast<char*>(&means[i * 3]), 12);
        f.read(reinterpret_cast<char*>(normals), 12);
        f.read(reinterpret_cast<char*>(&dc[i * 3]), 12);
        f.read(reinterpret_cast<char*>(&fr[(size_t)i * num_fr]), num_fr * 4);
        f.read(reinterpret_cast<char*>(&op[i]), 4);
        f.read(reinterpret_cast<char*>(&sc[i * 3]), 12);
        f.read(reinterpret_cast<char*>(&qt[i * 4]), 16);
    }
    if (!f) {
        set_error("PLY %s ends inside its vertex data", path);
        return MSPLAT_ERR_ARG;
    }
    if (keep_crs) {
        for (int i = 0; i < n; i++)
            for (int j = 0; j < 3; j++) means[i * 3 + j] = (means[i * 3 + j] - translation[j]) * scale;
        for (size_t i = 0; i < sc.size(); i++) sc[i] = std::log(scale * std::exp(sc[i]));
    }
    // [3, bases] -> [bases, 3]
    for (int i = 0; i < n; i++)
        for (int ch = 0; ch < 3; ch++)
            for (int b = 0; b < fr_bases; b++)
                rest[(size_t)i * num_fr + b * 3 + ch] = fr[(size_t)i * num_fr + ch * fr_bases + b];
    const std::vector<float>* src[kGroups] = {&means, &sc, &qt, &dc, &rest, &op};
    for (int g = 0; g < kGroups; g++)
        if ((rc = store(params[g], src[g]->data(), src[g]->size()))) return rc;
    return st;
}

}  // extern "C"
