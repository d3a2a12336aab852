// image_decode.cu -- training images from disk into HBM as float RGB.
//
// Replaces the reference's imreadRGB (core/src/loaders/image_io.cpp:12-56),
// which decodes through CoreGraphics into RGBA8 with the alpha channel
// skipped and converts to float v / 255.  Here:
//   JPEG  nvJPEG decodes on the GPU (interleaved RGB bytes in HBM);
//   PNG   a host decoder (zlib inflate + scanline unfiltering, all bit
//         depths, colour types and Adam7 interlacing) and one upload;
// and a kernel turns the bytes into floats on the device
// (msplat_bytes_to_rgb).  An RGBA PNG is composited over black, as drawing
// it into CoreGraphics' opaque RGBX context does; 16-bit samples keep their
// high byte.  Other formats are rejected with MSPLAT_ERR_ARG.
//
// nvJPEG is opened with dlopen on first use, so the engine library loads
// where it is absent; a JPEG then fails with a clear error.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvjpeg.h>
#include <zlib.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/msplat_engine.h"
#include "engine.h"

namespace msp {
namespace {

bool read_file(const char* path, std::vector<unsigned char>& out)
{
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    const long len = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    out.resize(len > 0 ? (size_t)len : 0);
    const bool ok = len >= 0 && std::fread(out.data(), 1, out.size(), f) == out.size();
    std::fclose(f);
    return ok;
}

uint32_t be32(const unsigned char* p)
{
    return ((uint32_t)p[0] << 24) | ((uint32_t)p[1] << 16) | ((uint32_t)p[2] << 8) | p[3];
}

bool is_png(const std::vector<unsigned char>& d)
{
    static const unsigned char sig[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1a, '\n'};
    return d.size() >= 8 && std::memcmp(d.data(), sig, 8) == 0;
}

bool is_jpeg(const std::vector<unsigned char>& d)
{
    return d.size() >= 3 && d[0] == 0xFF && d[1] == 0xD8 && d[2] == 0xFF;
}

// ---- PNG --------------------------------------------------------------------

struct Png {
    int w = 0, h = 0, depth = 0, color = 0, interlace = 0;
    std::vector<unsigned char> palette;  // RGB triples
    std::vector<unsigned char> idat;
};

int png_channels(int color)
{
    switch (color) {
        case 0: return 1;  // grey
        case 2: return 3;  // RGB
        case 3: return 1;  // palette index
        case 4: return 2;  // grey + alpha
        case 6: return 4;  // RGBA
        default: return 0;
    }
}

bool png_parse(const std::vector<unsigned char>& d, Png& p, std::string& err, bool header_only)
{
    size_t off = 8;
    bool have_ihdr = false;
    while (off + 8 <= d.size()) {
        const uint32_t len = be32(&d[off]);
        const char* type = reinterpret_cast<const char*>(&d[off + 4]);
        if (off + 12 + (size_t)len > d.size()) {
            err = "truncated PNG chunk";
            return false;
        }
        const unsigned char* body = &d[off + 8];
        if (!std::memcmp(type, "IHDR", 4) && len >= 13) {
            p.w = (int)be32(body);
            p.h = (int)be32(body + 4);
            p.depth = body[8];
            p.color = body[9];
            p.interlace = body[12];
            have_ihdr = true;
            if (header_only) return true;
        } else if (!std::memcmp(type, "PLTE", 4)) {
            p.palette.assign(body, body + len);
        } else if (!std::memcmp(type, "IDAT", 4)) {
            p.idat.insert(p.idat.end(), body, body + len);
        } else if (!std::memcmp(type, "IEND", 4)) {
            break;
        }
        off += 12 + (size_t)len;
    }
    if (!have_ihdr || p.w <= 0 || p.h <= 0) {
        err = "PNG without a valid IHDR";
        return false;
    }
    const int ch = png_channels(p.color);
    const int dp = p.depth;
    const bool depth_ok = (p.color == 0 && (dp == 1 || dp == 2 || dp == 4 || dp == 8 || dp == 16)) ||
                          (p.color == 3 && (dp == 1 || dp == 2 || dp == 4 || dp == 8)) ||
                          ((p.color == 2 || p.color == 4 || p.color == 6) && (dp == 8 || dp == 16));
    if (!ch || !depth_ok || p.interlace > 1) {
        err = "unsupported PNG colour type / bit depth / interlace";
        return false;
    }
    if (p.color == 3 && p.palette.size() < 3) {
        err = "palette PNG without PLTE";
        return false;
    }
    return true;
}

unsigned char paeth(int a, int b, int c)
{
    const int p = a + b - c;
    const int pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
    if (pa <= pb && pa <= pc) return (unsigned char)a;
    if (pb <= pc) return (unsigned char)b;
    return (unsigned char)c;
}

// Reverses the scanline filters of one (sub)image in place; `rows` rows of
// `stride` bytes, each preceded by its filter byte.
bool unfilter(unsigned char* data, int rows, size_t stride, int bpp, std::vector<unsigned char>& out)
{
    out.assign((size_t)rows * stride, 0);
    for (int y = 0; y < rows; y++) {
        const unsigned char* in = data + (size_t)y * (stride + 1);
        const int f = in[0];
        in++;
        unsigned char* cur = &out[(size_t)y * stride];
        const unsigned char* prev = y ? &out[(size_t)(y - 1) * stride] : nullptr;
        for (size_t i = 0; i < stride; i++) {
            const int a = i >= (size_t)bpp ? cur[i - bpp] : 0;
            const int b = prev ? prev[i] : 0;
            const int c = (prev && i >= (size_t)bpp) ? prev[i - bpp] : 0;
            int v = in[i];
            switch (f) {
                case 0: break;
                case 1: v += a; break;
                case 2: v += b; break;
                case 3: v += (a + b) >> 1; break;
                case 4: v += paeth(a, b, c); break;
                default: return false;
            }
            cur[i] = (unsigned char)v;
        }
    }
    return true;
}

// Sample `i` of a row of packed samples, expanded to 8 bits.
inline int sample8(const unsigned char* row, int i, int depth, bool palette)
{
    if (depth == 8) return row[i];
    if (depth == 16) return row[2 * i];  // high byte
    const int per_byte = 8 / depth;
    const int shift = 8 - depth * (1 + i % per_byte);
    const int v = (row[i / per_byte] >> shift) & ((1 << depth) - 1);
    return palette ? v : v * 255 / ((1 << depth) - 1);
}

// Decodes to interleaved bytes with `channels_out` = 1 (grey) or 3 (RGB).
bool png_decode(const std::vector<unsigned char>& file, std::vector<unsigned char>& pix, int& w,
                int& h, int& channels_out, std::string& err)
{
    Png p;
    if (!png_parse(file, p, err, false)) return false;
    w = p.w;
    h = p.h;
    const int ch = png_channels(p.color);
    const int bits = ch * p.depth;
    const int bpp = std::max(1, bits / 8);
    // Adam7 pass origins and steps; a non-interlaced image is one pass
    static const int ax0[7] = {0, 4, 0, 2, 0, 1, 0}, ay0[7] = {0, 0, 4, 0, 2, 0, 1};
    static const int adx[7] = {8, 8, 4, 4, 2, 2, 1}, ady[7] = {8, 8, 8, 4, 4, 2, 2};
    const int passes = p.interlace ? 7 : 1;
    size_t raw_size = 0;
    int pw[7], ph[7];
    for (int k = 0; k < passes; k++) {
        pw[k] = p.interlace ? (w - ax0[k] + adx[k] - 1) / adx[k] : w;
        ph[k] = p.interlace ? (h - ay0[k] + ady[k] - 1) / ady[k] : h;
        if (pw[k] > 0 && ph[k] > 0) raw_size += (size_t)ph[k] * (1 + ((size_t)pw[k] * bits + 7) / 8);
    }
    std::vector<unsigned char> raw(raw_size);
    uLongf got = (uLongf)raw_size;
    if (uncompress(raw.data(), &got, p.idat.data(), (uLong)p.idat.size()) != Z_OK || got != raw_size) {
        err = "PNG image data does not inflate to the expected size";
        return false;
    }
    const bool alpha = p.color == 4 || p.color == 6;
    const bool colour = p.color == 2 || p.color == 3 || p.color == 6;
    channels_out = colour ? 3 : 1;
    pix.assign((size_t)w * h * channels_out, 0);
    size_t off = 0;
    std::vector<unsigned char> rows;
    for (int k = 0; k < passes; k++) {
        if (pw[k] <= 0 || ph[k] <= 0) continue;
        const size_t stride = ((size_t)pw[k] * bits + 7) / 8;
        if (!unfilter(&raw[off], ph[k], stride, bpp, rows)) {
            err = "bad PNG filter type";
            return false;
        }
        off += (size_t)ph[k] * (stride + 1);
        for (int y = 0; y < ph[k]; y++) {
            const unsigned char* row = &rows[(size_t)y * stride];
            const int oy = p.interlace ? ay0[k] + y * ady[k] : y;
            for (int x = 0; x < pw[k]; x++) {
                const int ox = p.interlace ? ax0[k] + x * adx[k] : x;
                int c[3], a = 255;
                if (p.color == 3) {
                    const int idx = sample8(row, x, p.depth, true);
                    if ((size_t)idx * 3 + 2 >= p.palette.size()) {
                        err = "PNG palette index out of range";
                        return false;
                    }
                    for (int j = 0; j < 3; j++) c[j] = p.palette[idx * 3 + j];
                } else {
                    for (int j = 0; j < (colour ? 3 : 1); j++) c[j] = sample8(row, x * ch + j, p.depth, false);
                    if (alpha) a = sample8(row, x * ch + ch - 1, p.depth, false);
                }
                unsigned char* o = &pix[((size_t)oy * w + ox) * channels_out];
                for (int j = 0; j < channels_out; j++)
                    o[j] = (unsigned char)(alpha ? (c[j] * a + 127) / 255 : c[j]);
            }
        }
    }
    return true;
}

// ---- nvJPEG (dlopen) --------------------------------------------------------------

struct NvJpeg {
    bool tried = false;
    void* so = nullptr;
    nvjpegHandle_t handle = nullptr;
    nvjpegJpegState_t state = nullptr;
    decltype(&nvjpegCreateSimple) create = nullptr;
    decltype(&nvjpegJpegStateCreate) state_create = nullptr;
    decltype(&nvjpegGetImageInfo) info = nullptr;
    decltype(&nvjpegDecode) decode = nullptr;
    std::string err;
};

NvJpeg& nvjpeg()
{
    static NvJpeg j;
    if (j.tried) return j;
    j.tried = true;
    j.so = dlopen("libnvjpeg.so.12", RTLD_NOW | RTLD_LOCAL);
    if (!j.so) j.so = dlopen("libnvjpeg.so", RTLD_NOW | RTLD_LOCAL);
    if (!j.so) {
        j.err = "libnvjpeg is not available";
        return j;
    }
    j.create = (decltype(j.create))dlsym(j.so, "nvjpegCreateSimple");
    j.state_create = (decltype(j.state_create))dlsym(j.so, "nvjpegJpegStateCreate");
    j.info = (decltype(j.info))dlsym(j.so, "nvjpegGetImageInfo");
    j.decode = (decltype(j.decode))dlsym(j.so, "nvjpegDecode");
    if (!j.create || !j.state_create || !j.info || !j.decode) {
        j.err = "libnvjpeg lacks the simple decode API";
        j.decode = nullptr;
        return j;
    }
    if (j.create(&j.handle) != NVJPEG_STATUS_SUCCESS ||
        j.state_create(j.handle, &j.state) != NVJPEG_STATUS_SUCCESS) {
        j.err = "nvjpeg initialisation failed";
        j.decode = nullptr;
    }
    return j;
}

std::mutex g_decode_mu;         // one decode at a time (nvJPEG state, staging buffer)
unsigned char* g_stage = nullptr;
size_t g_stage_bytes = 0;

int stage(size_t bytes)
{
    if (bytes <= g_stage_bytes) return MSPLAT_OK;
    if (g_stage) cudaFree(g_stage);
    g_stage = nullptr;
    g_stage_bytes = 0;
    if (cudaMalloc(&g_stage, bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("image staging buffer of %zu bytes: out of device memory", bytes);
        return MSPLAT_ERR_CUDA;
    }
    g_stage_bytes = bytes;
    return MSPLAT_OK;
}

int jpeg_size(NvJpeg& j, const std::vector<unsigned char>& d, int* w, int* h)
{
    int comps = 0;
    nvjpegChromaSubsampling_t sub;
    int ws[NVJPEG_MAX_COMPONENT], hs[NVJPEG_MAX_COMPONENT];
    if (j.info(j.handle, d.data(), d.size(), &comps, &sub, ws, hs) != NVJPEG_STATUS_SUCCESS) {
        set_error("nvjpeg cannot read the JPEG header");
        return MSPLAT_ERR_ARG;
    }
    *w = ws[0];
    *h = hs[0];
    return MSPLAT_OK;
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_image_info(const char* path, int* width, int* height)
{
    std::vector<unsigned char> d;
    if (!path || !read_file(path, d)) {
        set_error("Failed to load image: %s", path ? path : "(null)");
        return MSPLAT_ERR_ARG;
    }
    int w = 0, h = 0;
    if (is_png(d)) {
        Png p;
        std::string err;
        if (!png_parse(d, p, err, true)) {
            set_error("%s: %s", path, err.c_str());
            return MSPLAT_ERR_ARG;
        }
        w = p.w;
        h = p.h;
    } else if (is_jpeg(d)) {
        std::lock_guard<std::mutex> lk(g_decode_mu);
        NvJpeg& j = nvjpeg();
        if (!j.decode) {
            set_error("%s: %s", path, j.err.c_str());
            return MSPLAT_ERR_CUDA;
        }
        int rc = jpeg_size(j, d, &w, &h);
        if (rc) return rc;
    } else {
        set_error("Failed to decode image (not PNG or JPEG): %s", path);
        return MSPLAT_ERR_ARG;
    }
    if (width) *width = w;
    if (height) *height = h;
    return MSPLAT_OK;
}

int msplat_image_decode(const char* path, float* dst, long long capacity_floats, int* width,
                        int* height)
{
    std::vector<unsigned char> d;
    if (!path || !dst || !read_file(path, d)) {
        set_error("Failed to load image: %s", path ? path : "(null)");
        return MSPLAT_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(g_decode_mu);
    int rc;
    {
        std::lock_guard<std::mutex> elk(engine_mutex());
        rc = engine_init();
    }
    if (rc) return rc;
    cudaStream_t s = engine_stream();
    int w = 0, h = 0, ch = 3;
    if (is_png(d)) {
        std::vector<unsigned char> pix;
        std::string err;
        if (!png_decode(d, pix, w, h, ch, err)) {
            set_error("%s: %s", path, err.c_str());
            return MSPLAT_ERR_ARG;
        }
        if ((long long)w * h * 3 > capacity_floats) {
            set_error("%s: %dx%d image does not fit the %lld floats given", path, w, h, capacity_floats);
            return MSPLAT_ERR_ARG;
        }
        if ((rc = stage(pix.size()))) return rc;
        if (cudaMemcpyAsync(g_stage, pix.data(), pix.size(), cudaMemcpyHostToDevice, s) != cudaSuccess) {
            set_error("%s: upload failed", path);
            return MSPLAT_ERR_CUDA;
        }
    } else if (is_jpeg(d)) {
        NvJpeg& j = nvjpeg();
        if (!j.decode) {
            set_error("%s: %s", path, j.err.c_str());
            return MSPLAT_ERR_CUDA;
        }
        if ((rc = jpeg_size(j, d, &w, &h))) return rc;
        if ((long long)w * h * 3 > capacity_floats) {
            set_error("%s: %dx%d image does not fit the %lld floats given", path, w, h, capacity_floats);
            return MSPLAT_ERR_ARG;
        }
        if ((rc = stage((size_t)w * h * 3))) return rc;
        nvjpegImage_t out{};
        out.channel[0] = g_stage;
        out.pitch[0] = (size_t)w * 3;
        const nvjpegStatus_t st = j.decode(j.handle, j.state, d.data(), d.size(), NVJPEG_OUTPUT_RGBI,
                                           &out, s);
        if (st != NVJPEG_STATUS_SUCCESS) {
            set_error("%s: nvjpeg decode failed (status %d)", path, (int)st);
            return MSPLAT_ERR_ARG;
        }
        ch = 3;
    } else {
        set_error("Failed to decode image (not PNG or JPEG): %s", path);
        return MSPLAT_ERR_ARG;
    }
    if ((rc = msplat_bytes_to_rgb(g_stage, w, h, ch, dst))) return rc;
    // the staging buffer and the host bytes are reused by the next call
    if (cudaStreamSynchronize(s) != cudaSuccess) {
        set_error("%s: decode failed on the device", path);
        return MSPLAT_ERR_CUDA;
    }
    if (width) *width = w;
    if (height) *height = h;
    return MSPLAT_OK;
}

}  // extern "C"
