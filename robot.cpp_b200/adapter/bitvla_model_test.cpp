// bitvla_model_test.cpp -- checks of the robotcpp::Model adapter (run by tests/test_robotcpp_adapter.py).
//   --cpu : observation -> engine input conversion and its error paths (no GPU needed);
//   --gpu : make_bitvla_model + predict() against b2s_bitvla_predict of the same inputs, bit for bit.
// Prints one line per failed check and "OK" at the end; the exit status is the number of failures.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "b2s.h"
#include "bitvla_model.h"

namespace {

int failures = 0;
#define CHECK(cond, what)                                          \
    do {                                                           \
        if (!(cond)) {                                             \
            std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, what); \
            ++failures;                                            \
        }                                                          \
    } while (0)

std::vector<uint8_t> random_bytes(size_t n, uint32_t seed) {
    std::mt19937 g(seed);
    std::vector<uint8_t> v(n);
    for (auto &b : v) b = (uint8_t)(g() & 0xFF);
    return v;
}

robotcpp::observation one_image(const uint8_t *data, int w, int h, int c, int stride, const std::string &task) {
    robotcpp::observation o;
    robotcpp::model_image im;
    im.name = "cam0";
    im.data = data;
    im.width = w;
    im.height = h;
    im.channels = c;
    im.stride_bytes = stride;
    o.images.push_back(im);
    o.task = task;
    return o;
}

void cpu_checks() {
    b2s_bitvla_config cfg;
    b2s_bitvla_default_config(&cfg);
    const int S = cfg.image_size;
    std::vector<uint8_t> img, img2;
    std::vector<int32_t> tok, tok2;
    std::string err;
    // Tight RGB and the same pixels with padded rows (stride_bytes honoured).
    const auto rgb = random_bytes((size_t)S * S * 3, 1);
    CHECK(b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, "ids:5,6,7"), cfg, img, tok, err),
          err.c_str());
    CHECK(img == rgb, "tight RGB copied unchanged");
    CHECK(tok.size() == (size_t)cfg.n_text && tok[0] == 5 && tok[1] == 6 && tok[2] == 7 && tok[3] == 0, "ids parsed");
    const int stride = S * 3 + 40;
    std::vector<uint8_t> padded((size_t)S * stride, 0xAB);
    for (int y = 0; y < S; ++y) std::memcpy(&padded[(size_t)y * stride], &rgb[(size_t)y * S * 3], (size_t)S * 3);
    CHECK(b2s_robotcpp::observation_to_inputs(one_image(padded.data(), S, S, 3, stride, "ids:5,6,7"), cfg, img2, tok2,
                                              err),
          err.c_str());
    CHECK(img2 == rgb && tok2 == tok, "stride_bytes honoured");
    // RGBA drops alpha; grey replicates.
    std::vector<uint8_t> rgba((size_t)S * S * 4);
    for (size_t i = 0; i < (size_t)S * S; ++i) {
        std::memcpy(&rgba[i * 4], &rgb[i * 3], 3);
        rgba[i * 4 + 3] = 7;
    }
    CHECK(b2s_robotcpp::observation_to_inputs(one_image(rgba.data(), S, S, 4, 0, ""), cfg, img2, tok2, err), err.c_str());
    CHECK(img2 == rgb, "RGBA -> RGB");
    const auto grey = random_bytes((size_t)S * S, 2);
    CHECK(b2s_robotcpp::observation_to_inputs(one_image(grey.data(), S, S, 1, 0, ""), cfg, img2, tok2, err), err.c_str());
    bool rep = true;
    for (size_t i = 0; i < (size_t)S * S; ++i) rep &= img2[i * 3] == grey[i] && img2[i * 3 + 1] == grey[i] && img2[i * 3 + 2] == grey[i];
    CHECK(rep, "grey replicated to RGB");
    // Resizing: a constant image stays constant; a 2x image of 2x2 blocks maps back to its block values.
    std::vector<uint8_t> flat((size_t)100 * 60 * 3, 77);
    CHECK(b2s_robotcpp::observation_to_inputs(one_image(flat.data(), 100, 60, 3, 0, ""), cfg, img2, tok2, err), err.c_str());
    bool cst = img2.size() == (size_t)S * S * 3;
    for (uint8_t v : img2) cst &= v == 77;
    CHECK(cst, "constant image resized to a constant image");
    // Hashed prompt: deterministic, in range, task-dependent; empty task = the default task.
    std::vector<int32_t> ta, tb, tc;
    b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, "pick up the red cup"), cfg, img2, ta, err);
    b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, "pick up the red cup"), cfg, img2, tb, err);
    b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, "open the drawer"), cfg, img2, tc, err);
    bool inr = true;
    for (int32_t t : ta) inr &= t >= 0 && t < cfg.vocab;
    CHECK(ta == tb && ta != tc && inr, "hashed prompt tokens");
    std::vector<int32_t> td, te;
    b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, ""), cfg, img2, td, err);
    b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, b2s_robotcpp::kDefaultTask), cfg, img2, te, err);
    CHECK(td == te, "empty task uses the default task");
    // Errors.
    robotcpp::observation none;
    CHECK(!b2s_robotcpp::observation_to_inputs(none, cfg, img2, tok2, err) && err.find("one image") != std::string::npos,
          "no image rejected");
    auto two = one_image(rgb.data(), S, S, 3, 0, "");
    two.images.push_back(two.images[0]);
    CHECK(!b2s_robotcpp::observation_to_inputs(two, cfg, img2, tok2, err), "two images rejected");
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(nullptr, S, S, 3, 0, ""), cfg, img2, tok2, err) &&
              err.find("null") != std::string::npos,
          "null data rejected");
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 2, 0, ""), cfg, img2, tok2, err) &&
              err.find("channels") != std::string::npos,
          "2 channels rejected");
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, S * 3 - 1, ""), cfg, img2, tok2, err) &&
              err.find("stride") != std::string::npos,
          "short stride rejected");
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), 0, S, 3, 0, ""), cfg, img2, tok2, err),
          "zero width rejected");
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, "ids:1,128256"), cfg, img2, tok2, err) &&
              err.find("outside") != std::string::npos,
          "out-of-vocabulary id rejected");
    std::string many = "ids:";
    for (int i = 0; i <= cfg.n_text; ++i) many += std::to_string(i) + ",";
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, many), cfg, img2, tok2, err),
          "too many ids rejected");
    CHECK(!b2s_robotcpp::observation_to_inputs(one_image(rgb.data(), S, S, 3, 0, "ids:1,x"), cfg, img2, tok2, err),
          "bad id rejected");
}

void gpu_checks() {
    robotcpp::model_args args;
    args.noise_seed = 1234;
    std::unique_ptr<robotcpp::Model> model;
    std::string err;
    CHECK(b2s_robotcpp::make_bitvla_model(args, model, err), err.c_str());
    if (!model) return;
    CHECK(std::string(model->type()) == "bitvla", "type()");
    b2s_bitvla_config cfg;
    b2s_bitvla_default_config(&cfg);
    const int S = cfg.image_size, A = cfg.action_chunk * cfg.action_dim;
    const auto rgb = random_bytes((size_t)S * S * 3, 9);
    const int stride = S * 3 + 24;
    std::vector<uint8_t> padded((size_t)S * stride, 0x11);
    for (int y = 0; y < S; ++y) std::memcpy(&padded[(size_t)y * stride], &rgb[(size_t)y * S * 3], (size_t)S * 3);
    std::string task = "ids:";
    std::vector<int32_t> tok((size_t)cfg.n_text);
    for (int i = 0; i < cfg.n_text; ++i) {
        tok[(size_t)i] = (int32_t)((i * 7919 + 13) % cfg.vocab);
        task += std::to_string(tok[(size_t)i]) + ",";
    }
    robotcpp::model_result res;
    const auto obs = one_image(padded.data(), S, S, 3, stride, task);
    CHECK(model->predict(obs, res, err), err.c_str());
    CHECK(res.chunk_size == cfg.action_chunk && res.action_dim == cfg.action_dim && (int)res.actions.size() == A,
          "result shape");
    bool have_total = false;
    for (const auto &m : res.metrics) have_total |= m.name == "model_total_ms" && m.value > 0.0;
    CHECK(have_total, "stage timings in metrics");
    // The same observation through the library's own entry point.
    b2s_bitvla *ref = nullptr;
    CHECK(b2s_bitvla_create(&cfg, 1234, 1, &ref) == B2S_OK, b2s_last_error());
    std::vector<float> act((size_t)A, NAN);
    CHECK(b2s_bitvla_predict(ref, 1, rgb.data(), tok.data(), act.data(), nullptr) == B2S_OK, b2s_last_error());
    CHECK(std::memcmp(act.data(), res.actions.data(), sizeof(float) * (size_t)A) == 0,
          "predict() equals b2s_bitvla_predict bit for bit");
    robotcpp::model_result res2;
    CHECK(model->predict(obs, res2, err) && res2.actions == res.actions, "repeatable");
    robotcpp::observation bad;
    CHECK(!model->predict(bad, res2, err) && res2.actions.empty(), "error path through predict()");
    b2s_bitvla_free(ref);
}

}  // namespace

int main(int argc, char **argv) {
    const std::string mode = argc > 1 ? argv[1] : "--cpu";
    if (mode == "--cpu") {
        cpu_checks();
    } else if (mode == "--gpu") {
        gpu_checks();
    } else {
        std::printf("usage: %s --cpu | --gpu\n", argv[0]);
        return 2;
    }
    if (!failures) std::printf("OK\n");
    return failures;
}
