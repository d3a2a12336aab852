// dataset.cu -- the real-data front end: dataset loaders (COLMAP, Nerfstudio,
// Polycam), point clouds, pose normalisation, train/test splits, and the
// ground-truth images resident in HBM with their downscaled forms.
//
// Reference counterparts:
//   inputDataFromX            core/src/input_data.cpp:195-217 (format dispatch)
//   loaders::loadColmap       core/src/loaders/load_colmap.cpp:9-164
//   loaders::loadNerfstudio   core/src/loaders/load_nerfstudio.cpp:10-72
//   loaders::loadPolycam      core/src/loaders/load_polycam.cpp:10-95
//   readPly / readColmapPoints core/src/loaders/load_ply.cpp:6-205
//   autoScaleAndCenter        core/src/input_data.cpp:79-123
//   getCameras / splitTrainTest core/src/input_data.cpp:127-160
//   Camera::loadImage / getImage / getGPUImage core/src/input_data.cpp:17-75
//
// Where the reference keeps each training image on the host and uploads a
// copy per downscale factor, this keeps the decoded image in device memory
// from the start: decode (image_decode.cu), resize and undistort
// (kernels_image.cu) all run on the GPU and the pyramid levels are made from
// the resident full image on first use.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <random>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace fs = std::filesystem;

namespace msp {
namespace {

// ---- a small JSON reader (objects, arrays, strings, numbers, literals) ---------

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    bool is_int = false;
    long long inum = 0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;

    const Json* get(const std::string& k) const
    {
        if (kind != Obj) return nullptr;
        for (auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
    bool contains(const std::string& k) const { return get(k) != nullptr; }
    float as_float() const
    {
        if (kind != Num) throw std::runtime_error("JSON value is not a number");
        return is_int ? (float)inum : (float)num;
    }
    int as_int() const
    {
        if (kind != Num) throw std::runtime_error("JSON value is not a number");
        return is_int ? (int)inum : (int)num;
    }
    // nlohmann's value(key, default): the member converted, or the default
    float value(const std::string& k, float dflt) const
    {
        const Json* v = get(k);
        return v ? v->as_float() : dflt;
    }
    int value(const std::string& k, int dflt) const
    {
        const Json* v = get(k);
        return v ? v->as_int() : dflt;
    }
    std::string value(const std::string& k, const char* dflt) const
    {
        const Json* v = get(k);
        if (!v) return dflt;
        if (v->kind != Str) throw std::runtime_error("JSON value is not a string");
        return v->str;
    }
};

struct JsonParser {
    const std::string& s;
    size_t i = 0;
    explicit JsonParser(const std::string& text) : s(text) {}

    [[noreturn]] void fail(const char* what)
    {
        throw std::runtime_error(std::string("JSON parse error: ") + what + " at offset " +
                                 std::to_string(i));
    }
    void ws()
    {
        while (i < s.size() && std::isspace((unsigned char)s[i])) i++;
    }
    Json parse()
    {
        Json v = value();
        ws();
        if (i != s.size()) fail("trailing characters");
        return v;
    }
    Json value()
    {
        ws();
        if (i >= s.size()) fail("unexpected end");
        const char c = s[i];
        Json v;
        if (c == '{') {
            v.kind = Json::Obj;
            i++;
            ws();
            if (i < s.size() && s[i] == '}') {
                i++;
                return v;
            }
            for (;;) {
                ws();
                if (i >= s.size() || s[i] != '"') fail("expected a key");
                std::string k = string();
                ws();
                if (i >= s.size() || s[i] != ':') fail("expected ':'");
                i++;
                v.obj.emplace_back(std::move(k), value());
                ws();
                if (i < s.size() && s[i] == ',') {
                    i++;
                    continue;
                }
                if (i < s.size() && s[i] == '}') {
                    i++;
                    return v;
                }
                fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v.kind = Json::Arr;
            i++;
            ws();
            if (i < s.size() && s[i] == ']') {
                i++;
                return v;
            }
            for (;;) {
                v.arr.push_back(value());
                ws();
                if (i < s.size() && s[i] == ',') {
                    i++;
                    continue;
                }
                if (i < s.size() && s[i] == ']') {
                    i++;
                    return v;
                }
                fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v.kind = Json::Str;
            v.str = string();
            return v;
        }
        if (!s.compare(i, 4, "true")) {
            i += 4;
            v.kind = Json::Bool;
            v.b = true;
            return v;
        }
        if (!s.compare(i, 5, "false")) {
            i += 5;
            v.kind = Json::Bool;
            return v;
        }
        if (!s.compare(i, 4, "null")) {
            i += 4;
            return v;
        }
        // number
        const size_t start = i;
        if (s[i] == '-') i++;
        bool integral = true;
        while (i < s.size() && (std::isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' ||
                                s[i] == 'E' || s[i] == '+' || s[i] == '-')) {
            if (s[i] == '.' || s[i] == 'e' || s[i] == 'E') integral = false;
            i++;
        }
        if (i == start) fail("unexpected character");
        const std::string tok = s.substr(start, i - start);
        v.kind = Json::Num;
        v.num = std::strtod(tok.c_str(), nullptr);
        if (integral) {
            v.is_int = true;
            v.inum = std::strtoll(tok.c_str(), nullptr, 10);
        }
        return v;
    }
    std::string string()
    {
        std::string out;
        i++;  // opening quote
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c != '\\') {
                out += c;
                continue;
            }
            if (i >= s.size()) fail("bad escape");
            const char e = s[i++];
            switch (e) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {
                    if (i + 4 > s.size()) fail("bad \\u escape");
                    unsigned cp = (unsigned)std::strtoul(s.substr(i, 4).c_str(), nullptr, 16);
                    i += 4;
                    if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' &&
                        s[i + 1] == 'u') {
                        const unsigned lo = (unsigned)std::strtoul(s.substr(i + 2, 4).c_str(), nullptr, 16);
                        i += 6;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    if (cp < 0x80) {
                        out += (char)cp;
                    } else if (cp < 0x800) {
                        out += (char)(0xC0 | (cp >> 6));
                        out += (char)(0x80 | (cp & 0x3F));
                    } else if (cp < 0x10000) {
                        out += (char)(0xE0 | (cp >> 12));
                        out += (char)(0x80 | ((cp >> 6) & 0x3F));
                        out += (char)(0x80 | (cp & 0x3F));
                    } else {
                        out += (char)(0xF0 | (cp >> 18));
                        out += (char)(0x80 | ((cp >> 12) & 0x3F));
                        out += (char)(0x80 | ((cp >> 6) & 0x3F));
                        out += (char)(0x80 | (cp & 0x3F));
                    }
                    break;
                }
                default: out += e; break;  // \" \\ \/
            }
        }
        if (i >= s.size()) fail("unterminated string");
        i++;
        return out;
    }
};

Json read_json(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Cannot open " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    return JsonParser(text).parse();
}

// ---- dataset model ---------------------------------------------------------------

struct DevImage {
    float* ptr = nullptr;
    int w = 0, h = 0;
};

struct Cam {
    int width = 0, height = 0;
    float fx = 0, fy = 0, cx = 0, cy = 0;
    float k1 = 0, k2 = 0, k3 = 0, p1 = 0, p2 = 0;
    float c2w[16] = {};
    std::string path;
    DevImage image;                   // Camera::image, resident
    std::map<int, DevImage> pyramid;  // Camera::getImage(k) levels, resident

    bool distorted() const { return k1 != 0 || k2 != 0 || k3 != 0 || p1 != 0 || p2 != 0; }
};

struct Points {
    std::vector<float> xyz;
    std::vector<unsigned char> rgb;
    long long count = 0;
};

}  // namespace
}  // namespace msp

struct MsplatData {
    std::vector<msp::Cam> cams;
    float scale = 1.0f;
    float translation[3] = {0, 0, 0};
    msp::Points points;
    ~MsplatData()
    {
        for (auto& c : cams) {
            if (c.image.ptr) cudaFree(c.image.ptr);
            for (auto& kv : c.pyramid) cudaFree(kv.second.ptr);
        }
    }
};

namespace msp {
namespace {

// ---- point clouds ---------------------------------------------------------------

enum class PlyT { F32, F64, U8, U16, I32, Unknown };

PlyT ply_type(const std::string& t)
{
    if (t == "float" || t == "float32") return PlyT::F32;
    if (t == "double" || t == "float64") return PlyT::F64;
    if (t == "uchar" || t == "uint8") return PlyT::U8;
    if (t == "ushort" || t == "uint16") return PlyT::U16;
    if (t == "int" || t == "int32") return PlyT::I32;
    return PlyT::Unknown;
}

int ply_size(PlyT t)
{
    switch (t) {
        case PlyT::F32: return 4;
        case PlyT::F64: return 8;
        case PlyT::U8: return 1;
        case PlyT::U16: return 2;
        case PlyT::I32: return 4;
        default: return 0;
    }
}

// A point cloud PLY (ascii or binary little endian): x y z and, when all
// three are present, red green blue (default grey 128).  As in the
// reference, every property after the "element vertex" line counts toward
// the vertex record.
Points read_points_ply(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Cannot open PLY file: " + path);
    std::string line;
    std::getline(f, line);
    if (line.find("ply") == std::string::npos) throw std::runtime_error("Not a PLY file: " + path);
    bool binary = false, ascii = false;
    int nv = 0;
    struct Prop {
        std::string name;
        PlyT type;
        int offset;
    };
    std::vector<Prop> props;
    int rec = 0;
    while (std::getline(f, line)) {
        if (line == "end_header") break;
        std::istringstream iss(line);
        std::string tok;
        iss >> tok;
        if (tok == "format") {
            std::string fmt;
            iss >> fmt;
            binary = fmt == "binary_little_endian";
            ascii = fmt == "ascii";
        } else if (tok == "element") {
            std::string name;
            iss >> name;
            if (name == "vertex") iss >> nv;
        } else if (tok == "property" && nv > 0) {
            std::string type, name;
            iss >> type >> name;
            const PlyT t = ply_type(type);
            props.push_back({name, t, rec});
            rec += ply_size(t);
        }
    }
    if (nv == 0) throw std::runtime_error("PLY has no vertices");
    if (!binary && !ascii)
        throw std::runtime_error("Unsupported PLY format (need ascii or binary_little_endian)");
    auto find = [&](const char* name) {
        for (size_t i = 0; i < props.size(); i++)
            if (props[i].name == name) return (int)i;
        return -1;
    };
    const int ix = find("x"), iy = find("y"), iz = find("z");
    const int ir = find("red"), ig = find("green"), ib = find("blue");
    if (ix < 0 || iy < 0 || iz < 0) throw std::runtime_error("PLY missing x/y/z properties");
    Points pts;
    pts.count = nv;
    pts.xyz.resize((size_t)nv * 3);
    pts.rgb.assign((size_t)nv * 3, 128);
    const bool colour = ir >= 0 && ig >= 0 && ib >= 0;
    if (binary) {
        std::vector<char> buf(rec);
        auto rf = [&](int pi) -> float {
            const Prop& p = props[pi];
            if (p.type == PlyT::F32) {
                float v;
                std::memcpy(&v, &buf[p.offset], 4);
                return v;
            }
            if (p.type == PlyT::F64) {
                double v;
                std::memcpy(&v, &buf[p.offset], 8);
                return (float)v;
            }
            return 0.0f;
        };
        auto ru8 = [&](int pi) -> unsigned char {
            const Prop& p = props[pi];
            if (p.type == PlyT::U8) return (unsigned char)buf[p.offset];
            if (p.type == PlyT::U16) {
                uint16_t v;
                std::memcpy(&v, &buf[p.offset], 2);
                return (unsigned char)(v >> 8);
            }
            if (p.type == PlyT::F32) {
                float v;
                std::memcpy(&v, &buf[p.offset], 4);
                return (unsigned char)(v * 255.0f);
            }
            return 128;
        };
        for (int i = 0; i < nv; i++) {
            f.read(buf.data(), rec);
            pts.xyz[i * 3 + 0] = rf(ix);
            pts.xyz[i * 3 + 1] = rf(iy);
            pts.xyz[i * 3 + 2] = rf(iz);
            if (colour) {
                pts.rgb[i * 3 + 0] = ru8(ir);
                pts.rgb[i * 3 + 1] = ru8(ig);
                pts.rgb[i * 3 + 2] = ru8(ib);
            }
        }
    } else {
        for (int i = 0; i < nv; i++) {
            std::getline(f, line);
            std::istringstream iss(line);
            std::vector<std::string> toks;
            std::string t;
            while (iss >> t) toks.push_back(t);
            auto at = [&](int k) -> const std::string& {
                if (k >= (int)toks.size()) throw std::runtime_error("PLY ascii row too short");
                return toks[k];
            };
            pts.xyz[i * 3 + 0] = std::stof(at(ix));
            pts.xyz[i * 3 + 1] = std::stof(at(iy));
            pts.xyz[i * 3 + 2] = std::stof(at(iz));
            if (colour) {
                const float rv = std::stof(at(ir)), gv = std::stof(at(ig)), bv = std::stof(at(ib));
                const bool flt = props[ir].type == PlyT::F32 || props[ir].type == PlyT::F64;
                pts.rgb[i * 3 + 0] = (unsigned char)(flt ? rv * 255.0f : rv);
                pts.rgb[i * 3 + 1] = (unsigned char)(flt ? gv * 255.0f : gv);
                pts.rgb[i * 3 + 2] = (unsigned char)(flt ? bv * 255.0f : bv);
            }
        }
    }
    return pts;
}

// COLMAP points3D.bin: id, xyz (f64), rgb (u8), error (f64), track.
Points read_colmap_points(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Cannot open points3D.bin: " + path);
    uint64_t n = 0;
    f.read(reinterpret_cast<char*>(&n), 8);
    Points pts;
    pts.count = (long long)n;
    pts.xyz.resize(n * 3);
    pts.rgb.resize(n * 3);
    for (uint64_t i = 0; i < n; i++) {
        uint64_t id, track;
        double xyz[3], err;
        unsigned char rgb[3];
        f.read(reinterpret_cast<char*>(&id), 8);
        f.read(reinterpret_cast<char*>(xyz), 24);
        f.read(reinterpret_cast<char*>(rgb), 3);
        f.read(reinterpret_cast<char*>(&err), 8);
        f.read(reinterpret_cast<char*>(&track), 8);
        f.seekg((std::streamoff)(track * 8), std::ios::cur);
        for (int j = 0; j < 3; j++) {
            pts.xyz[i * 3 + j] = (float)xyz[j];
            pts.rgb[i * 3 + j] = rgb[j];
        }
    }
    if (!f) throw std::runtime_error("points3D.bin is truncated: " + path);
    return pts;
}

// ---- COLMAP ---------------------------------------------------------------------

struct ColmapCam {
    int model = 0, width = 0, height = 0;
    float fx = 0, fy = 0, cx = 0, cy = 0, k1 = 0, k2 = 0, p1 = 0, p2 = 0;
};

struct ColmapImage {
    uint32_t cam = 0;
    double q[4] = {1, 0, 0, 0};  // w x y z, world to camera
    double t[3] = {0, 0, 0};
    std::string name;
};

std::unordered_map<uint32_t, ColmapCam> read_colmap_cameras(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Cannot open " + path);
    uint64_t n = 0;
    f.read(reinterpret_cast<char*>(&n), 8);
    std::unordered_map<uint32_t, ColmapCam> out;
    for (uint64_t i = 0; i < n; i++) {
        uint32_t id, model;
        uint64_t w, h;
        f.read(reinterpret_cast<char*>(&id), 4);
        f.read(reinterpret_cast<char*>(&model), 4);
        f.read(reinterpret_cast<char*>(&w), 8);
        f.read(reinterpret_cast<char*>(&h), 8);
        ColmapCam c;
        c.model = (int)model;
        c.width = (int)w;
        c.height = (int)h;
        auto rd = [&]() {
            double v = 0;
            f.read(reinterpret_cast<char*>(&v), 8);
            return (float)v;
        };
        // parameter lists per model: SIMPLE_PINHOLE f cx cy; PINHOLE fx fy cx cy;
        // SIMPLE_RADIAL f cx cy k; RADIAL f cx cy k1 k2; OPENCV fx fy cx cy k1 k2 p1 p2
        switch (c.model) {
            case 0: c.fx = c.fy = rd(); c.cx = rd(); c.cy = rd(); break;
            case 1: c.fx = rd(); c.fy = rd(); c.cx = rd(); c.cy = rd(); break;
            case 2: c.fx = c.fy = rd(); c.cx = rd(); c.cy = rd(); c.k1 = rd(); break;
            case 3: c.fx = c.fy = rd(); c.cx = rd(); c.cy = rd(); c.k1 = rd(); c.k2 = rd(); break;
            case 4:
                c.fx = rd(); c.fy = rd(); c.cx = rd(); c.cy = rd();
                c.k1 = rd(); c.k2 = rd(); c.p1 = rd(); c.p2 = rd();
                break;
            default:
                throw std::runtime_error("Unsupported COLMAP camera model: " + std::to_string(c.model));
        }
        out[id] = c;
    }
    if (!f) throw std::runtime_error("cameras.bin is truncated: " + path);
    return out;
}

std::vector<ColmapImage> read_colmap_images(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) throw std::runtime_error("Cannot open " + path);
    uint64_t n = 0;
    f.read(reinterpret_cast<char*>(&n), 8);
    std::vector<ColmapImage> out;
    out.reserve(n);
    for (uint64_t i = 0; i < n; i++) {
        ColmapImage im;
        uint32_t id;
        f.read(reinterpret_cast<char*>(&id), 4);
        f.read(reinterpret_cast<char*>(im.q), 32);
        f.read(reinterpret_cast<char*>(im.t), 24);
        f.read(reinterpret_cast<char*>(&im.cam), 4);
        char ch;
        while (f.read(&ch, 1) && ch != '\0') im.name += ch;
        uint64_t n2d = 0;
        f.read(reinterpret_cast<char*>(&n2d), 8);
        f.seekg((std::streamoff)(n2d * 24), std::ios::cur);
        out.push_back(std::move(im));
    }
    if (!f) throw std::runtime_error("images.bin is truncated: " + path);
    return out;
}

// World-to-camera (unit quaternion w x y z, translation) -> camera-to-world,
// row-major 4x4, with the camera's y and z axes flipped (OpenCV -> OpenGL).
// The rotation is formed in double and rounded to float, the inverse
// translation -R^T t in float, as the reference does.
void colmap_pose(const double q[4], const double t[3], float out[16])
{
    double w = q[0], x = q[1], y = q[2], z = q[3];
    const double n = std::sqrt(w * w + x * x + y * y + z * z);
    w /= n;
    x /= n;
    y /= n;
    z /= n;
    const float R[9] = {
        (float)(1 - 2 * (y * y + z * z)), (float)(2 * (x * y - w * z)), (float)(2 * (x * z + w * y)),
        (float)(2 * (x * y + w * z)), (float)(1 - 2 * (x * x + z * z)), (float)(2 * (y * z - w * x)),
        (float)(2 * (x * z - w * y)), (float)(2 * (y * z + w * x)), (float)(1 - 2 * (x * x + y * y)),
    };
    const float tf[3] = {(float)t[0], (float)t[1], (float)t[2]};
    for (int r = 0; r < 3; r++) {
        // row r of R^T is column r of R
        const float a = R[r], b = R[3 + r], c = R[6 + r];
        out[r * 4 + 0] = a;
        out[r * 4 + 1] = -b;
        out[r * 4 + 2] = -c;
        out[r * 4 + 3] = -(a * tf[0] + b * tf[1] + c * tf[2]);
    }
    out[12] = out[13] = out[14] = 0;
    out[15] = 1;
}

void auto_scale_and_center(MsplatData& d);

void load_colmap(MsplatData& d, const std::string& root_s, const std::string& image_src)
{
    const fs::path root(root_s);
    const std::string sparse = fs::exists(root / "cameras.bin") ? root_s : (root / "sparse" / "0").string();
    const std::string images = !image_src.empty()           ? image_src
                               : fs::exists(root / "images") ? (root / "images").string()
                                                             : root_s;
    auto cams = read_colmap_cameras(sparse + "/cameras.bin");
    auto ims = read_colmap_images(sparse + "/images.bin");
    std::sort(ims.begin(), ims.end(),
              [](const ColmapImage& a, const ColmapImage& b) { return a.name < b.name; });
    for (auto& im : ims) {
        auto it = cams.find(im.cam);
        if (it == cams.end()) continue;
        const ColmapCam& cc = it->second;
        Cam c;
        c.width = cc.width;
        c.height = cc.height;
        c.fx = cc.fx;
        c.fy = cc.fy;
        c.cx = cc.cx;
        c.cy = cc.cy;
        c.k1 = cc.k1;
        c.k2 = cc.k2;
        c.p1 = cc.p1;
        c.p2 = cc.p2;
        c.path = images + "/" + im.name;
        colmap_pose(im.q, im.t, c.c2w);
        d.cams.push_back(std::move(c));
    }
    const std::string pts = sparse + "/points3D.bin";
    if (fs::exists(pts))
        d.points = read_colmap_points(pts);
    else if (fs::exists(sparse + "/points3D.ply"))
        d.points = read_points_ply(sparse + "/points3D.ply");
    auto_scale_and_center(d);
}

// ---- Nerfstudio / Polycam ----------------------------------------------------------

std::string with_image_ext(const std::string& p)
{
    if (fs::exists(p)) return p;
    for (const char* ext : {".png", ".jpg", ".jpeg", ".JPG"})
        if (fs::exists(p + ext)) return p + ext;
    return p;
}

void read_matrix(const Json& tm, float out[16])
{
    if (tm.kind != Json::Arr || tm.arr.size() < 4) throw std::runtime_error("bad transform_matrix");
    for (int r = 0; r < 4; r++) {
        if (tm.arr[r].kind != Json::Arr || tm.arr[r].arr.size() < 4)
            throw std::runtime_error("bad transform_matrix row");
        for (int c = 0; c < 4; c++) out[r * 4 + c] = tm.arr[r].arr[c].as_float();
    }
}

void load_nerfstudio(MsplatData& d, const std::string& root_s)
{
    const fs::path root(root_s);
    const Json j = read_json((root / "transforms.json").string());
    const int gw = j.value("w", 0), gh = j.value("h", 0);
    const float gfx = j.value("fl_x", 0.0f), gfy = j.value("fl_y", 0.0f);
    const float gcx = j.value("cx", 0.0f), gcy = j.value("cy", 0.0f);
    const float gk1 = j.value("k1", 0.0f), gk2 = j.value("k2", 0.0f), gk3 = j.value("k3", 0.0f);
    const float gp1 = j.value("p1", 0.0f), gp2 = j.value("p2", 0.0f);
    const Json* frames = j.get("frames");
    if (!frames || frames->kind != Json::Arr) throw std::runtime_error("transforms.json has no frames");
    for (const Json& fr : frames->arr) {
        Cam c;
        c.width = fr.value("w", gw);
        c.height = fr.value("h", gh);
        c.fx = fr.value("fl_x", gfx);
        c.fy = fr.value("fl_y", gfy);
        c.cx = fr.value("cx", gcx);
        c.cy = fr.value("cy", gcy);
        c.k1 = fr.value("k1", gk1);
        c.k2 = fr.value("k2", gk2);
        c.k3 = fr.value("k3", gk3);
        c.p1 = fr.value("p1", gp1);
        c.p2 = fr.value("p2", gp2);
        const Json* fp = fr.get("file_path");
        if (!fp || fp->kind != Json::Str) throw std::runtime_error("frame without file_path");
        const bool as_is = !fp->str.empty() && (fp->str[0] == '/' || fp->str[0] == '.');
        c.path = as_is ? with_image_ext(fp->str) : with_image_ext((root / fp->str).string());
        const Json* tm = fr.get("transform_matrix");
        if (!tm) throw std::runtime_error("frame without transform_matrix");
        read_matrix(*tm, c.c2w);
        d.cams.push_back(std::move(c));
    }
    std::sort(d.cams.begin(), d.cams.end(), [](const Cam& a, const Cam& b) { return a.path < b.path; });
    if (const Json* pp = j.get("ply_file_path")) {
        if (pp->kind != Json::Str) throw std::runtime_error("ply_file_path is not a string");
        std::string p = pp->str;
        if (p.empty() || p[0] != '/') p = (root / p).string();
        if (fs::exists(p)) d.points = read_points_ply(p);
    }
    if (d.points.count == 0) {
        for (const char* p : {"sparse/0/points3D.ply", "points3D.ply"}) {
            const std::string path = (root / p).string();
            if (fs::exists(path)) {
                d.points = read_points_ply(path);
                break;
            }
        }
    }
    auto_scale_and_center(d);
}

std::string polycam_image(const fs::path& dir, const std::string& stem)
{
    for (const char* ext : {".png", ".jpg", ".jpeg", ".JPG"}) {
        const fs::path p = dir / (stem + ext);
        if (fs::exists(p)) return p.string();
    }
    return (dir / (stem + ".png")).string();
}

void load_polycam(MsplatData& d, const std::string& root_s)
{
    const fs::path root(root_s);
    const fs::path kf = root / "keyframes" / "corrected_cameras";
    const fs::path imgs = root / "keyframes" / "corrected_images";
    if (fs::exists(kf)) {
        std::vector<fs::path> files;
        for (auto& e : fs::directory_iterator(kf))
            if (e.path().extension() == ".json") files.push_back(e.path());
        std::sort(files.begin(), files.end());
        for (auto& jp : files) {
            const Json j = read_json(jp.string());
            Cam c;
            c.width = j.value("width", 0);
            c.height = j.value("height", 0);
            c.fx = j.value("fx", 0.0f);
            c.fy = j.value("fy", 0.0f);
            c.cx = j.value("cx", (float)c.width / 2.0f);
            c.cy = j.value("cy", (float)c.height / 2.0f);
            float R[9], T[3];
            for (int r = 0; r < 3; r++)
                for (int k = 0; k < 3; k++)
                    R[r * 3 + k] = j.value("R_" + std::to_string(r) + std::to_string(k), 0.0f);
            T[0] = j.value("t_20", 0.0f);
            T[1] = j.value("t_21", 0.0f);
            T[2] = j.value("t_22", 0.0f);
            // first row kept, second and third negated (OpenGL y/z flip)
            const float sgn[3] = {1.f, -1.f, -1.f};
            for (int r = 0; r < 3; r++) {
                for (int k = 0; k < 3; k++) c.c2w[r * 4 + k] = sgn[r] == 1.f ? R[r * 3 + k] : -R[r * 3 + k];
                c.c2w[r * 4 + 3] = sgn[r] == 1.f ? T[r] : -T[r];
            }
            c.c2w[12] = c.c2w[13] = c.c2w[14] = 0;
            c.c2w[15] = 1;
            c.path = polycam_image(imgs, jp.stem().string());
            d.cams.push_back(std::move(c));
        }
    } else {
        const Json j = read_json((root / "cameras.json").string());
        const Json* frames = j.contains("frames") ? j.get("frames") : &j;
        const std::vector<Json>* list = nullptr;
        std::vector<Json> values;
        if (frames->kind == Json::Arr) {
            list = &frames->arr;
        } else if (frames->kind == Json::Obj) {  // iterating an object visits its values
            for (auto& kv : frames->obj) values.push_back(kv.second);
            list = &values;
        } else {
            throw std::runtime_error("cameras.json: no frames");
        }
        for (const Json& fr : *list) {
            Cam c;
            c.width = fr.value("width", 0);
            c.height = fr.value("height", 0);
            c.fx = fr.value("fx", 0.0f);
            c.fy = fr.value("fy", 0.0f);
            c.cx = fr.value("cx", (float)c.width / 2.0f);
            c.cy = fr.value("cy", (float)c.height / 2.0f);
            if (const Json* tm = fr.get("transform_matrix")) read_matrix(*tm, c.c2w);
            c.path = fr.value("file_path", "");
            if (!c.path.empty() && c.path[0] != '/') c.path = (root / c.path).string();
            d.cams.push_back(std::move(c));
        }
    }
    for (const char* p : {"keyframes/point_cloud.ply", "point_cloud.ply", "sparse.ply"}) {
        const std::string path = (root / p).string();
        if (fs::exists(path)) {
            d.points = read_points_ply(path);
            break;
        }
    }
    auto_scale_and_center(d);
}

// Centre the camera positions on their mean and scale them into [-1, 1]
// (by the largest absolute coordinate); the point cloud follows.
void auto_scale_and_center(MsplatData& d)
{
    if (d.cams.empty()) return;
    float mean[3] = {0, 0, 0};
    for (auto& c : d.cams) {
        mean[0] += c.c2w[3];
        mean[1] += c.c2w[7];
        mean[2] += c.c2w[11];
    }
    const int n = (int)d.cams.size();
    for (int k = 0; k < 3; k++) {
        mean[k] /= (float)n;
        d.translation[k] = mean[k];
    }
    for (auto& c : d.cams) {
        c.c2w[3] -= mean[0];
        c.c2w[7] -= mean[1];
        c.c2w[11] -= mean[2];
    }
    float max_abs = 0;
    for (auto& c : d.cams) {
        max_abs = std::max(max_abs, std::abs(c.c2w[3]));
        max_abs = std::max(max_abs, std::abs(c.c2w[7]));
        max_abs = std::max(max_abs, std::abs(c.c2w[11]));
    }
    d.scale = max_abs > 0 ? 1.0f / max_abs : 1.0f;
    for (auto& c : d.cams) {
        c.c2w[3] *= d.scale;
        c.c2w[7] *= d.scale;
        c.c2w[11] *= d.scale;
    }
    for (long long i = 0; i < d.points.count; i++)
        for (int k = 0; k < 3; k++)
            d.points.xyz[i * 3 + k] = (d.points.xyz[i * 3 + k] - mean[k]) * d.scale;
}

// ---- device images -------------------------------------------------------------------

int dev_alloc(DevImage& im, int w, int h)
{
    im.w = w;
    im.h = h;
    if (cudaMalloc(&im.ptr, (size_t)w * h * 3 * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        im.ptr = nullptr;
        set_error("out of device memory for a %dx%d image", w, h);
        return MSPLAT_ERR_CUDA;
    }
    return MSPLAT_OK;
}

void dev_free(DevImage& im)
{
    if (im.ptr) cudaFree(im.ptr);
    im = DevImage{};
}

// Camera::loadImage: decode, fit the intrinsics to the decoded size,
// downscale by `df` (> 1), undistort and crop.  The result stays in HBM.
int load_image(Cam& c, float df)
{
    int rw = 0, rh = 0;
    int rc = msplat_image_info(c.path.c_str(), &rw, &rh);
    if (rc) return rc;
    DevImage raw;
    if ((rc = dev_alloc(raw, rw, rh))) return rc;
    if ((rc = msplat_image_decode(c.path.c_str(), raw.ptr, (long long)rw * rh * 3, &rw, &rh))) {
        dev_free(raw);
        return rc;
    }
    if (c.width > 0 && c.height > 0 && (rw != c.width || rh != c.height)) {
        const float sx = (float)rw / (float)c.width, sy = (float)rh / (float)c.height;
        c.fx *= sx;
        c.fy *= sy;
        c.cx *= sx;
        c.cy *= sy;
        c.width = rw;
        c.height = rh;
    } else if (c.width == 0 || c.height == 0) {
        c.width = rw;
        c.height = rh;
    }
    if (df > 1.0f) {
        const int nw = (int)((float)c.width / df), nh = (int)((float)c.height / df);
        DevImage small;
        if ((rc = dev_alloc(small, nw, nh)) ||
            (rc = msplat_resize_area(raw.ptr, raw.w, raw.h, small.ptr, nw, nh))) {
            dev_free(raw);
            dev_free(small);
            return rc;
        }
        cudaStreamSynchronize(engine_stream());
        dev_free(raw);
        raw = small;
        const float s = 1.0f / df;
        c.fx *= s;
        c.fy *= s;
        c.cx *= s;
        c.cy *= s;
        c.width = nw;
        c.height = nh;
    }
    if (c.distorted()) {
        int roi[4];
        if ((rc = msplat_undistort_roi(raw.w, raw.h, c.fx, c.fy, c.cx, c.cy, c.k1, c.k2, c.p1, c.p2,
                                       c.k3, roi))) {
            dev_free(raw);
            return rc;
        }
        DevImage und;
        if ((rc = dev_alloc(und, roi[2], roi[3])) ||
            (rc = msplat_undistort(raw.ptr, raw.w, raw.h, c.fx, c.fy, c.cx, c.cy, c.k1, c.k2, c.p1,
                                   c.p2, c.k3, roi, und.ptr))) {
            dev_free(raw);
            dev_free(und);
            return rc;
        }
        cudaStreamSynchronize(engine_stream());
        dev_free(raw);
        raw = und;
        c.cx -= (float)roi[0];
        c.cy -= (float)roi[1];
        c.width = roi[2];
        c.height = roi[3];
        c.k1 = c.k2 = c.k3 = c.p1 = c.p2 = 0;
    }
    dev_free(c.image);
    for (auto& kv : c.pyramid) dev_free(kv.second);
    c.pyramid.clear();
    c.image = raw;
    return MSPLAT_OK;
}

int catch_all(const std::exception& e)
{
    set_error("%s", e.what());
    return MSPLAT_ERR_ARG;
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_dataset_open(const char* path, const char* colmap_image_path, MsplatData** out)
{
    if (!path || !out) {
        set_error("msplat_dataset_open: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    *out = nullptr;
    try {
        auto d = std::make_unique<MsplatData>();
        const fs::path root(path);
        if (fs::exists(root / "transforms.json"))
            load_nerfstudio(*d, path);
        else if (fs::exists(root / "cameras.bin") || fs::exists(root / "sparse" / "0" / "cameras.bin"))
            load_colmap(*d, path, colmap_image_path ? colmap_image_path : "");
        else if (fs::exists(root / "keyframes" / "corrected_cameras") || fs::exists(root / "cameras.json"))
            load_polycam(*d, path);
        else
            throw std::runtime_error(std::string("Unrecognized dataset format in: ") + path +
                                     " (supported: COLMAP (cameras.bin), Nerfstudio (transforms.json), "
                                     "Polycam (keyframes/))");
        *out = d.release();
        return MSPLAT_OK;
    } catch (const std::exception& e) {
        return catch_all(e);
    }
}

void msplat_dataset_close(MsplatData* d) { delete d; }

int msplat_dataset_num_cameras(const MsplatData* d) { return d ? (int)d->cams.size() : MSPLAT_ERR_ARG; }

int msplat_dataset_camera(const MsplatData* d, int i, MsplatCameraInfo* out)
{
    if (!d || !out || i < 0 || i >= (int)d->cams.size()) {
        set_error("msplat_dataset_camera: index %d out of range", i);
        return MSPLAT_ERR_ARG;
    }
    const Cam& c = d->cams[i];
    out->width = c.width;
    out->height = c.height;
    out->fx = c.fx;
    out->fy = c.fy;
    out->cx = c.cx;
    out->cy = c.cy;
    out->k1 = c.k1;
    out->k2 = c.k2;
    out->k3 = c.k3;
    out->p1 = c.p1;
    out->p2 = c.p2;
    std::memcpy(out->cam_to_world, c.c2w, sizeof(c.c2w));
    return MSPLAT_OK;
}

const char* msplat_dataset_camera_path(const MsplatData* d, int i)
{
    if (!d || i < 0 || i >= (int)d->cams.size()) return nullptr;
    return d->cams[i].path.c_str();
}

long long msplat_dataset_points(const MsplatData* d, const float** xyz, const unsigned char** rgb)
{
    if (!d) return MSPLAT_ERR_ARG;
    if (xyz) *xyz = d->points.xyz.data();
    if (rgb) *rgb = d->points.rgb.data();
    return d->points.count;
}

int msplat_dataset_transform(const MsplatData* d, float* scale, float* translation)
{
    if (!d) return MSPLAT_ERR_ARG;
    if (scale) *scale = d->scale;
    if (translation) std::memcpy(translation, d->translation, 3 * sizeof(float));
    return MSPLAT_OK;
}

int msplat_dataset_split(const MsplatData* d, int test_every, int* train_idx, int* n_train,
                         int* test_idx, int* n_test)
{
    if (!d || test_every <= 0) {
        set_error("msplat_dataset_split: invalid arguments");
        return MSPLAT_ERR_ARG;
    }
    int a = 0, b = 0;
    for (int i = 0; i < (int)d->cams.size(); i++) {
        if (i % test_every == 0) {
            if (test_idx) test_idx[b] = i;
            b++;
        } else {
            if (train_idx) train_idx[a] = i;
            a++;
        }
    }
    if (n_train) *n_train = a;
    if (n_test) *n_test = b;
    return MSPLAT_OK;
}

int msplat_dataset_validation_camera(const MsplatData* d, const char* val_image)
{
    if (!d || d->cams.empty()) {
        set_error("msplat_dataset_validation_camera: no cameras");
        return MSPLAT_ERR_ARG;
    }
    const std::string v = val_image ? val_image : "random";
    int idx = -1;
    if (v == "random") {
        std::mt19937 rng(42);
        idx = (int)(rng() % d->cams.size());
    } else {
        for (int i = 0; i < (int)d->cams.size(); i++)
            if (d->cams[i].path.find(v) != std::string::npos) {
                idx = i;
                break;
            }
    }
    return idx < 0 ? 0 : idx;
}

int msplat_dataset_load_images(MsplatData* d, float downscale_factor)
{
    if (!d) return MSPLAT_ERR_ARG;
    for (auto& c : d->cams) {
        int rc = load_image(c, downscale_factor);
        if (rc) return rc;
    }
    return MSPLAT_OK;
}

int msplat_dataset_load_image(MsplatData* d, int i, float downscale_factor)
{
    if (!d || i < 0 || i >= (int)d->cams.size()) {
        set_error("msplat_dataset_load_image: index %d out of range", i);
        return MSPLAT_ERR_ARG;
    }
    return load_image(d->cams[i], downscale_factor);
}

int msplat_dataset_gt(MsplatData* d, int i, int downscale, const float** dev_rgb, int* width,
                      int* height)
{
    if (!d || i < 0 || i >= (int)d->cams.size()) {
        set_error("msplat_dataset_gt: index %d out of range", i);
        return MSPLAT_ERR_ARG;
    }
    Cam& c = d->cams[i];
    if (!c.image.ptr) {
        set_error("msplat_dataset_gt: camera %d has no image loaded", i);
        return MSPLAT_ERR_ARG;
    }
    const DevImage* im = &c.image;
    if (downscale > 1) {
        auto it = c.pyramid.find(downscale);
        if (it == c.pyramid.end()) {
            DevImage s;
            const int nw = c.image.w / downscale, nh = c.image.h / downscale;
            int rc = dev_alloc(s, nw, nh);
            if (!rc) rc = msplat_resize_area(c.image.ptr, c.image.w, c.image.h, s.ptr, nw, nh);
            if (rc) {
                dev_free(s);
                return rc;
            }
            it = c.pyramid.emplace(downscale, s).first;
        }
        im = &it->second;
    }
    if (dev_rgb) *dev_rgb = im->ptr;
    if (width) *width = im->w;
    if (height) *height = im->h;
    return MSPLAT_OK;
}

long long msplat_dataset_device_bytes(const MsplatData* d)
{
    if (!d) return 0;
    long long b = 0;
    for (auto& c : d->cams) {
        b += (long long)c.image.w * c.image.h * 12;
        for (auto& kv : c.pyramid) b += (long long)kv.second.w * kv.second.h * 12;
    }
    return b;
}

}  // extern "C"
