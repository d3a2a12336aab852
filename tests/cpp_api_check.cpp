// The reference's C++ API (include/msplat_api.hpp) driven as an application
// would: load a dataset, train, evaluate, render, export, checkpoint and
// resume.  Built and run by tests/test_cpp_api.py; prints one line per
// check and exits non-zero on the first failure.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "msplat_api.hpp"

#define CHECK(cond)                                                       \
    do {                                                                  \
        if (!(cond)) {                                                    \
            std::fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
            return 1;                                                     \
        }                                                                 \
        std::printf("ok: %s\n", #cond);                                   \
    } while (0)

int main(int argc, char** argv)
{
    if (argc < 3) return 2;
    const std::string data = argv[1], out = argv[2];
    msplat::Dataset ds(data, 1.0f, true, 4);
    CHECK(ds.numTrain() == 6 && ds.numTest() == 2);
    msplat::Config cfg;
    cfg.iterations = 12;
    cfg.numDownscales = 0;
    msplat::Trainer t(ds, cfg);
    CHECK(t.iteration() == 0 && t.splatCount() == 400);
    msplat::Stats s = t.step();
    CHECK(s.iteration == 1 && s.splatCount == 400 && s.msPerStep >= 0.f);
    t.train(0);
    CHECK(t.iteration() == 12);
    msplat::EvalMetrics m = t.evaluate();
    CHECK(m.numTest == 2 && m.psnr > 0.f && m.ssim > 0.f && m.ssim < 1.f && m.l1 > 0.f);
    msplat::PixelBuffer img = t.render(0, false);
    CHECK(img.data != nullptr && img.width > 0 && img.height > 0);
    float pose[16];
    ds.cameraPose(1, pose);
    msplat::PixelBuffer img2 = t.renderFromPose(pose, 1);
    msplat::PixelBuffer img3 = t.render(1, false);
    bool same = img2.width == img3.width && img2.height == img3.height;
    for (int i = 0; same && i < img2.width * img2.height * 3; i++) same = img2.data[i] == img3.data[i];
    CHECK(same);
    int w = 0, h = 0;
    t.renderFromPoseToBuffer(pose, 1, nullptr, &w, &h);
    std::vector<uint8_t> rgba((size_t)w * h * 4);
    t.renderFromPoseToBuffer(pose, 1, rgba.data(), &w, &h);
    CHECK(w == img3.width && rgba[3] == 255 &&
          rgba[0] == (uint8_t)(std::min(std::max(img3.data[0], 0.f), 1.f) * 255.f));
    t.exportPly(out + "/scene.ply");
    t.exportSplat(out + "/scene.splat");
    t.saveCheckpoint(out + "/scene.msplat");
    msplat::Config cfg2 = cfg;
    cfg2.iterations = 15;
    msplat::Trainer t2(ds, cfg2);
    CHECK(t2.loadCheckpoint(out + "/scene.msplat") == 12 && t2.splatCount() == t.splatCount());
    t2.train(0);
    CHECK(t2.iteration() == 15);
    msplat::PixelBuffer moved = std::move(img);
    CHECK(moved.data != nullptr && img.data == nullptr);
    bool threw = false;
    try {
        msplat::Dataset bad(out + "/no-such-dataset", 1.0f, false, 8);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw);
    msplat::sync();
    return 0;
}
