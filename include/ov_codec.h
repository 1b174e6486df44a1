/*
 * ov_codec.h - C-ABI of the OmniVoice audio tokenizer on B200: the decoder
 * (residual-vector-quantized codes to 24 kHz float32 audio) and the encoder
 * (24 kHz audio to codes, for voice cloning).
 *
 * Replaces the decoding half of the reference's C++ class
 * gufo::models::omnivoice::Codec (codec.hpp:17-43):
 *   ov_codec_load          <- Codec::Load   (codec.cpp:114-193, decoder weights)
 *   ov_codec_decode        <- Codec::Decode (codec.cpp:195-262)
 * plus ov_codec_decode_device, which takes the codes and returns the audio
 * in device memory (the generator's codes never leave the GPU), and
 * ov_codec_create_synthetic (random-init weights of the same shapes).
 * The encoding half (voice cloning) is a separate handle:
 *   ov_codec_encoder_load  <- Codec::Load   (codec.cpp:188, LoadEncoder,
 *                             codec_encoder.cpp:72-247)
 *   ov_codec_encode        <- Codec::Encode (codec_encoder.cpp:249-458)
 * A codec is not thread-safe (codec.hpp:16); use one per GPU.
 */
#ifndef OV_CODEC_H_
#define OV_CODEC_H_

#include <stddef.h>
#include <stdint.h>

#include "ov_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ov_codec ov_codec;

/* The decoder's part of CodecConfig (config.hpp:41-72): codebooks,
 * entries and code width of the RVQ, the semantic and acoustic widths whose
 * sum is the quantizer's hidden size (codec.cpp:121-122), the DAC decoder's
 * first width (halved by every upsampling block) and strides, the output
 * sample rate.  frame_samples is the product of the strides. */
typedef struct {
  size_t codebooks;
  size_t codebook_size;
  size_t codebook_dim;
  size_t semantic_hidden;
  size_t latent_channels;
  size_t decoder_channels;
  size_t upsampling_ratios[8];
  size_t num_upsampling;
  uint32_t sample_rate;
} ov_codec_config;

/* Higgs Audio v2 tokenizer as OmniVoice ships it: 8 x 1024 codes of width 64,
 * 768 + 256 hidden, decoder 1024 channels, strides 8 5 4 2 3 (960 samples
 * per frame at 24 kHz). */
void ov_codec_default_config(ov_codec_config* config);

/* Loads the decoder tensors of `audio_tokenizer/model.safetensors` (float32,
 * the reference's names and shapes, codec.cpp:26-106,131-188) onto
 * `device`. */
int ov_codec_load(const ov_codec_config* config, const char* safetensors_path, int device,
                  ov_codec** codec);
/* Random-init weights of the configured shapes, generated from `seed`. */
int ov_codec_create_synthetic(const ov_codec_config* config, uint64_t seed, int device,
                              ov_codec** codec);
void ov_codec_free(ov_codec* codec);

size_t ov_codec_frame_samples(const ov_codec* codec);

/* codes: HOST int32 [codebooks][frames], each in [0, codebook_size);
 * audio: HOST float32 [frames * frame_samples].  Errors carry the
 * reference's "OmniVoice decode: " prefix. */
int ov_codec_decode(ov_codec* codec, const int32_t* codes, size_t frames, float* audio);

/* The same with DEVICE codes and audio, enqueued on `stream` (NULL: the
 * codec's own stream) without a host synchronisation; out-of-range codes
 * are clamped to entry 0 and reported by ov_take_device_errors. */
int ov_codec_decode_device(ov_codec* codec, const int32_t* codes, size_t frames, float* audio,
                           ov_stream_t stream);

/* ------------------------------------------------------------ encoder */

typedef struct ov_codec_encoder ov_codec_encoder;

/* The encoder's part of CodecConfig (config.hpp:30-72): the codec's rate
 * and quantizer, HuBERT (SemanticEncoderConfig: rate, widths, heads,
 * layers, the grouped positional convolution, layer-norm epsilon and the
 * feature extractor's convolutions) and the DAC encoder (AcousticConfig:
 * first width, doubled by every downsampling block, latent width and
 * strides).  The joint width of fc and the quantizer is hidden_size +
 * latent_channels; frame_samples is the product of the DAC strides. */
typedef struct {
  uint32_t sample_rate;
  size_t codebooks;
  size_t codebook_size;
  size_t codebook_dim;
  uint32_t semantic_sample_rate;
  size_t hidden_size;
  size_t intermediate_size;
  size_t heads;
  size_t layers;
  size_t position_kernel;
  size_t position_groups;
  float layer_norm_eps;
  size_t conv_channels[8];
  size_t conv_kernels[8];
  size_t conv_strides[8];
  size_t num_convs;
  size_t encoder_channels;
  size_t latent_channels;
  size_t downsampling_ratios[8];
  size_t num_downsampling;
} ov_codec_encoder_config;

/* Higgs Audio v2 tokenizer as OmniVoice ships it: HuBERT base (768 wide,
 * 12 layers of 12 heads, 3072 intermediate, 7 convolutions of 512 with
 * kernels 10 3 3 3 3 2 2 and strides 5 2 2 2 2 2 2 at 16 kHz, positional
 * kernel 128 in 16 groups), DAC encoder 64 channels with strides 8 5 4 2 3
 * to a 256-wide latent, 8 x 1024 codes of width 64 at 24 kHz. */
void ov_codec_encoder_default_config(ov_codec_encoder_config* config);
/* Loads the encoder tensors of `audio_tokenizer/model.safetensors` (float32,
 * the reference's names and shapes, codec_encoder.cpp:72-247, and the
 * quantizer's project_out for the decoded entries). */
int ov_codec_encoder_load(const ov_codec_encoder_config* config, const char* safetensors_path,
                          int device, ov_codec_encoder** encoder);
/* Random-init weights of the configured shapes, generated from `seed`. */
int ov_codec_encoder_create_synthetic(const ov_codec_encoder_config* config, uint64_t seed,
                                      int device, ov_codec_encoder** encoder);
void ov_codec_encoder_free(ov_codec_encoder* encoder);
size_t ov_codec_encoder_frame_samples(const ov_codec_encoder* encoder);

/* samples: HOST float32 mono at sample_rate, a whole number of frames;
 * codes: HOST int32 [codebooks][frames] with room for `capacity` values;
 * *frames receives the frame count.  Errors carry the reference's
 * "OmniVoice encode: " prefix (a partial frame, audio too short for the
 * semantic encoder). */
int ov_codec_encode(ov_codec_encoder* encoder, const float* samples, size_t count, int32_t* codes,
                    size_t capacity, size_t* frames);

#ifdef __cplusplus
}
#endif

#endif /* OV_CODEC_H_ */
