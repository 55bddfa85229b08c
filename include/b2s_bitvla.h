/* b2s_bitvla.h -- random-init BitVLA-shape forward on the B200 ternary kernels (C ABI).
 *
 * The reference has no BitVLA model (robotcpp::model_type lists smolvla and pi0 only,
 * src/models/model.h:10-13); this engine is the caller the i2_s mul_mat exists for. Its layer
 * structure follows the reference's own engines: the ViT block of src/models/smolvla/vision.cpp:305-345
 * (LayerNorm -> q/k/v -> softmax attention -> o + residual -> LayerNorm -> fc1 -> GELU -> fc2 + residual)
 * and the decoder layer of src/models/pi0/vlm.cpp:196-246 (RMSNorm -> q/k/v -> NEOX RoPE -> GQA
 * attention -> o + residual -> RMSNorm -> gate/up -> down + residual), with every linear layer a
 * ternary i2_s weight (BitNet b1.58: per-token int8 activations, sub-norms before o and down).
 *
 * One observation = one CHW fp32 image (image_size^2, values in [0,1]) and n_text token ids. The vision
 * tower turns the image into (image_size/patch)^2 tokens, a two-layer ternary connector maps them to the
 * decoder width, the text tokens are embedded, and the decoder runs a causal prefill over
 * n_patches + n_text tokens. Outputs: the final-RMSNorm hidden states of every token and an fp32 action
 * chunk (action_chunk x action_dim) read out of the last token by a linear head.
 *
 * Weights are random-init from a seed (no checkpoint exists); every parameter is a pure function of
 * (seed, tensor id, element index) -- see b2s_bitvla_param_bits -- so a CPU restatement regenerates the
 * identical model. A forward for a given batch size is captured once into a CUDA graph and replayed.
 * Weights and activation buffers live on the device current at b2s_bitvla_create.
 */
#ifndef B2S_BITVLA_H
#define B2S_BITVLA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2s_bitvla_config {
    int image_size;   /* 224 */
    int patch;        /* 14 -> 256 patches */
    int vit_layers;   /* 27 */
    int vit_hidden;   /* 1152 */
    int vit_ffn;      /* 4304 */
    int vit_heads;    /* 16 (head dim 72) */
    float vit_eps;    /* LayerNorm eps, 1e-6 */
    int conn_hidden;  /* connector hidden width, 2560 */
    int dec_layers;   /* 30 */
    int dec_hidden;   /* 2560 */
    int dec_ffn;      /* 6912 */
    int dec_heads;    /* 20 */
    int dec_kv_heads; /* 5 */
    int head_dim;     /* 128 */
    float rope_theta; /* 500000 */
    float dec_eps;    /* RMSNorm eps, 1e-5 */
    int vocab;        /* 128256 */
    int n_text;       /* 32 */
    int action_chunk; /* 8 */
    int action_dim;   /* 7 */
    int attention_tc;   /* 0 (default): the fixed-order fp32 attention kernel (b2s_attention), which the CPU
                           oracle repeats bit for bit, so the whole forward is bit-exact. 1: attention on the
                           tensor cores (b2s_attention_tc, 3xTF32 products, within 1e-5 of the oracle per
                           operator). The int8 act-quant between layers amplifies any rounding difference (a
                           2^-22 relative change of the input image moves the oracle's own outputs by several
                           percent), so with 1 the forward differs from the oracle by a few percent end to end. */
} b2s_bitvla_config;

typedef struct b2s_bitvla b2s_bitvla;

/* The BitVLA shape above. */
void b2s_bitvla_default_config(b2s_bitvla_config *cfg);

/* Tokens per observation in the decoder: (image_size/patch)^2 + n_text. */
int b2s_bitvla_seq_len(const b2s_bitvla_config *cfg);

/* Ternary multiply-accumulates x 2 per observation (the int8 ops the i2_s GEMMs execute). */
double b2s_bitvla_ternary_ops(const b2s_bitvla_config *cfg);

/* Parameter generator shared with the CPU restatement: 32 hash bits of element `idx` of tensor `tensor`.
 * Ternary weights: u = bits >> 8; u < 5033165 -> -1, u < 11744051 -> 0, else +1 (P(0) = 0.4);
 * fp32 parameters: lo + width * (u * 2^-24). */
uint32_t b2s_bitvla_param_bits(uint32_t seed, uint32_t tensor, uint32_t idx);

/* Builds the model on the current device, generating every weight from `seed`; max_batch observations
 * per forward. Returns B2S_OK or a b2s_status (see b2s_last_error()). */
int b2s_bitvla_create(const b2s_bitvla_config *cfg, uint32_t seed, int max_batch, b2s_bitvla **out);
void b2s_bitvla_free(b2s_bitvla *m);

/* Builds the model from a GGUF file (general.architecture "bitvla"; the shape from the bitvla.* keys,
 * the text-embedding seed from bitvla.token_embd.seed; ternary weights as I2_S tensors, type 36, in the
 * flattened i2_s layout with the fp32 scale in the 32-byte trailer; everything else F32). The tensor names
 * and keys are the ones robot.cpp_b200/b2s/gguf.py writes. This mirrors gguf_loader::load ->
 * parse_metadata -> bind_tensors (src/models/gguf_loader.cpp:9-162): i2_s bytes reach the device
 * unchanged and are repacked to padded rows there. A file written from seed S loads into the same model
 * as b2s_bitvla_create(..., S, ...). */
int b2s_bitvla_create_from_gguf(const char *path, int max_batch, b2s_bitvla **out);

/* The model's shape (the config it was built with, or the one read from its GGUF file). */
int b2s_bitvla_get_config(const b2s_bitvla *m, b2s_bitvla_config *cfg);

/* Device bytes held by the packed ternary weights / by all weights / by activation buffers. */
size_t b2s_bitvla_ternary_bytes(const b2s_bitvla *m);
size_t b2s_bitvla_weight_bytes(const b2s_bitvla *m);
size_t b2s_bitvla_activation_bytes(const b2s_bitvla *m);

/* Forward of `batch` observations (1 <= batch <= max_batch) on `stream`, all pointers device memory:
 * images [batch][3][image_size][image_size] fp32, tokens [batch][n_text] int32 in [0, vocab);
 * hidden [batch * seq_len][dec_hidden] fp32 (may be NULL); actions [batch][action_chunk * action_dim]
 * fp32 (may be NULL). The first call for a batch size captures the graph (not inside another capture). */
int b2s_bitvla_forward(b2s_bitvla *m, int batch, const float *images, const int32_t *tokens, float *hidden,
                       float *actions, void *stream);

/* The same from host memory (robotcpp::Model::predict shape): images [batch][H][W][3] uint8 (value/255),
 * tokens [batch][n_text]; writes actions to host memory [batch][action_chunk * action_dim]. Copies go
 * through the model's pinned staging buffers on `stream`; returns after the actions have arrived. */
int b2s_bitvla_predict(b2s_bitvla *m, int batch, const uint8_t *images_hwc, const int32_t *tokens,
                       float *actions, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* B2S_BITVLA_H */
