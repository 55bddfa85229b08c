// bitvla_model.h -- the BitVLA-shape engine of libb2s.so as a robotcpp::Model.
//
// Compiled against the reference's own interface header (src/models/model.h:64-72: Model::type, predict,
// reset; observation / model_image / model_result at :15-39), found through the include path the Makefile
// passes (ROBOTCPP_SRC); the header is not copied here. A maintainer registers it with one enum value and
// one factory branch (src/models/model.h:10-13, src/models/model_factory.cpp:8-19):
//     enum class model_type { smolvla, pi0, bitvla };
//     if (args.type == model_type::bitvla) return b2s_robotcpp::make_bitvla_model(args, out, error);
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "b2s_bitvla.h"
#include "models/model.h"

namespace b2s_robotcpp {

// The prompt used when an observation has no task text (the reference's SmolVLA default,
// src/models/smolvla/smolvla_model.cpp:98).
constexpr const char *kDefaultTask = "grab the block.";

// One observation in the engine's input form:
//   image: obs.images must hold exactly one image; data non-null; channels 1 (grey, replicated to RGB),
//     3 (RGB) or 4 (RGBA, alpha dropped); rows stride_bytes apart (0 means width * channels, smaller is an
//     error); any width x height, resized to image_size x image_size by bilinear interpolation with
//     half-pixel centres when it differs; written as HWC uint8 RGB.
//   tokens: a task of the form "ids:<id>,<id>,..." gives the token ids directly (each in [0, vocab), at most
//     n_text of them, the rest filled with id 0); any other task (empty means kDefaultTask) is mapped by a
//     byte-level hash (no tokenizer model exists for a random-init vocabulary): token i is FNV-1a over the
//     task's bytes followed by the four little-endian bytes of i, modulo vocab.
//   obs.state is not used by this model (BitVLA takes no proprioceptive input).
bool observation_to_inputs(const robotcpp::observation &obs, const b2s_bitvla_config &cfg,
                           std::vector<uint8_t> &image_hwc, std::vector<int32_t> &tokens, std::string &error);

class BitVLAModel final : public robotcpp::Model {
  public:
    ~BitVLAModel() override;
    const char *type() const override;
    // Actions of one observation (action_chunk x action_dim floats) with the stage timings in out.metrics:
    // preprocess_ms (host conversion), bitvla_ms (b2s_bitvla_predict: copies, graph replay, actions back),
    // model_total_ms.
    bool predict(const robotcpp::observation &obs, robotcpp::model_result &out, std::string &error) override;
    void reset() override {}

  private:
    friend bool make_bitvla_model(const robotcpp::model_args &, std::unique_ptr<robotcpp::Model> &, std::string &);
    BitVLAModel() = default;
    b2s_bitvla *model_ = nullptr;
    b2s_bitvla_config cfg_{};
};

// args.llm_path, when set, names a BitVLA GGUF file (b2s_bitvla_create_from_gguf); otherwise the
// random-init BitVLA shape is built from args.noise_seed (1234 when negative). The model lives on the
// current CUDA device.
bool make_bitvla_model(const robotcpp::model_args &args, std::unique_ptr<robotcpp::Model> &out, std::string &error);

}  // namespace b2s_robotcpp
