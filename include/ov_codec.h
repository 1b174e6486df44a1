/*
 * ov_codec.h - C-ABI of the OmniVoice audio tokenizer's decoder on B200:
 * residual-vector-quantized codes to 24 kHz float32 audio.
 *
 * Replaces the decoding half of the reference's C++ class
 * gufo::models::omnivoice::Codec (codec.hpp:17-43):
 *   ov_codec_load          <- Codec::Load   (codec.cpp:114-193, decoder weights)
 *   ov_codec_decode        <- Codec::Decode (codec.cpp:195-262)
 * plus ov_codec_decode_device, which takes the codes and returns the audio
 * in device memory (the generator's codes never leave the GPU), and
 * ov_codec_create_synthetic (random-init weights of the same shapes).
 * The encoder (Codec::Encode, voice cloning) is not part of this library.
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

#ifdef __cplusplus
}
#endif

#endif /* OV_CODEC_H_ */
