// bitvla_model.cpp -- robotcpp::Model adapter of the BitVLA-shape engine (see bitvla_model.h).
#include "bitvla_model.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "b2s.h"

namespace b2s_robotcpp {

namespace {

using Clock = std::chrono::steady_clock;

double ms_since(Clock::time_point t0) { return std::chrono::duration<double, std::milli>(Clock::now() - t0).count(); }

void add_metric(robotcpp::model_result &out, const char *name, double v) {
    robotcpp::model_metric m;
    m.name = name;
    m.value = v;
    out.metrics.push_back(m);
}

// RGB value of pixel (x, y) of the source image.
inline void src_rgb(const robotcpp::model_image &im, int stride, int x, int y, uint8_t rgb[3]) {
    const uint8_t *p = im.data + (size_t)y * (size_t)stride + (size_t)x * (size_t)im.channels;
    if (im.channels == 1) {
        rgb[0] = rgb[1] = rgb[2] = p[0];
    } else {
        rgb[0] = p[0];
        rgb[1] = p[1];
        rgb[2] = p[2];
    }
}

uint32_t fnv1a(const std::string &s, uint32_t i) {
    uint32_t h = 2166136261u;
    for (unsigned char c : s) h = (h ^ c) * 16777619u;
    for (int b = 0; b < 4; ++b) h = (h ^ ((i >> (8 * b)) & 0xFFu)) * 16777619u;
    return h;
}

}  // namespace

bool observation_to_inputs(const robotcpp::observation &obs, const b2s_bitvla_config &cfg,
                           std::vector<uint8_t> &image_hwc, std::vector<int32_t> &tokens, std::string &error) {
    if (obs.images.size() != 1) {
        error = "BitVLA takes exactly one image per observation (got " + std::to_string(obs.images.size()) + ")";
        return false;
    }
    const robotcpp::model_image &im = obs.images[0];
    if (im.data == nullptr) {
        error = "BitVLA image data is null";
        return false;
    }
    if (im.width <= 0 || im.height <= 0) {
        error = "BitVLA image has a non-positive size";
        return false;
    }
    if (im.channels != 1 && im.channels != 3 && im.channels != 4) {
        error = "BitVLA image must have 1, 3 or 4 channels (got " + std::to_string(im.channels) + ")";
        return false;
    }
    const int row = im.width * im.channels;
    const int stride = im.stride_bytes == 0 ? row : im.stride_bytes;
    if (stride < row) {
        error = "BitVLA image stride_bytes (" + std::to_string(im.stride_bytes) + ") is below width * channels";
        return false;
    }
    const int S = cfg.image_size;
    image_hwc.assign((size_t)S * S * 3, 0);
    if (im.width == S && im.height == S) {
        for (int y = 0; y < S; ++y)
            for (int x = 0; x < S; ++x) src_rgb(im, stride, x, y, &image_hwc[((size_t)y * S + x) * 3]);
    } else {  // bilinear, half-pixel centres, edge-clamped
        const float sx = (float)im.width / (float)S, sy = (float)im.height / (float)S;
        for (int y = 0; y < S; ++y) {
            const float fy = std::fmax(0.0f, ((float)y + 0.5f) * sy - 0.5f);
            const int y0 = std::min((int)fy, im.height - 1), y1 = std::min(y0 + 1, im.height - 1);
            const float wy = fy - (float)y0;
            for (int x = 0; x < S; ++x) {
                const float fx = std::fmax(0.0f, ((float)x + 0.5f) * sx - 0.5f);
                const int x0 = std::min((int)fx, im.width - 1), x1 = std::min(x0 + 1, im.width - 1);
                const float wx = fx - (float)x0;
                uint8_t a[3], b[3], c[3], d[3];
                src_rgb(im, stride, x0, y0, a);
                src_rgb(im, stride, x1, y0, b);
                src_rgb(im, stride, x0, y1, c);
                src_rgb(im, stride, x1, y1, d);
                for (int ch = 0; ch < 3; ++ch) {
                    const float top = (float)a[ch] + wx * ((float)b[ch] - (float)a[ch]);
                    const float bot = (float)c[ch] + wx * ((float)d[ch] - (float)c[ch]);
                    const float v = top + wy * (bot - top);
                    image_hwc[((size_t)y * S + x) * 3 + (size_t)ch] = (uint8_t)std::lround(std::fmin(255.0f, std::fmax(0.0f, v)));
                }
            }
        }
    }
    tokens.assign((size_t)cfg.n_text, 0);
    const std::string task = obs.task.empty() ? std::string(kDefaultTask) : obs.task;
    if (task.rfind("ids:", 0) == 0) {
        const char *p = task.c_str() + 4;
        int n = 0;
        while (*p) {
            while (*p == ' ' || *p == ',') ++p;
            if (!*p) break;
            char *end = nullptr;
            const long v = std::strtol(p, &end, 10);
            if (end == p) {
                error = "BitVLA task ids: not an integer at '" + std::string(p) + "'";
                return false;
            }
            if (v < 0 || v >= cfg.vocab) {
                error = "BitVLA token id " + std::to_string(v) + " outside [0, " + std::to_string(cfg.vocab) + ")";
                return false;
            }
            if (n >= cfg.n_text) {
                error = "BitVLA task has more than " + std::to_string(cfg.n_text) + " token ids";
                return false;
            }
            tokens[(size_t)n++] = (int32_t)v;
            p = end;
        }
    } else {
        for (int i = 0; i < cfg.n_text; ++i) tokens[(size_t)i] = (int32_t)(fnv1a(task, (uint32_t)i) % (uint32_t)cfg.vocab);
    }
    return true;
}

BitVLAModel::~BitVLAModel() { b2s_bitvla_free(model_); }

const char *BitVLAModel::type() const { return "bitvla"; }

bool BitVLAModel::predict(const robotcpp::observation &obs, robotcpp::model_result &out, std::string &error) {
    out = robotcpp::model_result{};
    if (model_ == nullptr) {
        error = "BitVLA model is not initialized";
        return false;
    }
    const Clock::time_point t0 = Clock::now();
    std::vector<uint8_t> img;
    std::vector<int32_t> tok;
    if (!observation_to_inputs(obs, cfg_, img, tok, error)) return false;
    const double pre_ms = ms_since(t0);
    const int A = cfg_.action_chunk * cfg_.action_dim;
    out.actions.assign((size_t)A, 0.0f);
    const Clock::time_point t1 = Clock::now();
    const int rc = b2s_bitvla_predict(model_, 1, img.data(), tok.data(), out.actions.data(), nullptr);
    if (rc != B2S_OK) {
        error = std::string("b2s_bitvla_predict failed: ") + b2s_last_error();
        out.actions.clear();
        return false;
    }
    out.chunk_size = cfg_.action_chunk;
    out.action_dim = cfg_.action_dim;
    add_metric(out, "preprocess_ms", pre_ms);
    add_metric(out, "bitvla_ms", ms_since(t1));
    add_metric(out, "model_total_ms", ms_since(t0));
    return true;
}

bool make_bitvla_model(const robotcpp::model_args &args, std::unique_ptr<robotcpp::Model> &out, std::string &error) {
    out.reset();
    std::unique_ptr<BitVLAModel> m(new (std::nothrow) BitVLAModel());
    if (!m) {
        error = "failed to allocate BitVLA model";
        return false;
    }
    int rc;
    if (!args.llm_path.empty()) {
        rc = b2s_bitvla_create_from_gguf(args.llm_path.c_str(), 1, &m->model_);
    } else {
        b2s_bitvla_config cfg;
        b2s_bitvla_default_config(&cfg);
        const uint32_t seed = args.noise_seed >= 0 ? (uint32_t)args.noise_seed : 1234u;
        rc = b2s_bitvla_create(&cfg, seed, 1, &m->model_);
    }
    if (rc != B2S_OK) {
        error = std::string("failed to initialize BitVLA model: ") + b2s_last_error();
        return false;
    }
    b2s_bitvla_get_config(m->model_, &m->cfg_);
    out = std::move(m);
    return true;
}

}  // namespace b2s_robotcpp
