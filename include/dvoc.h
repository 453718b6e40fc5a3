/*
 * dvoc.h -- C ABI of the B200-native (sm_100a) vocoder of dots.tts: the
 * decode path of the BigVGAN AudioVAE (nanovllm_dots/models/dots/native/
 * vocoder/bigvgan.py), latent frames in, 48 kHz audio out.
 *
 * The reference decodes one request at a time from Python:
 *   - one-shot: AudioVAE.inference_from_latents(z, do_sample=False)
 *     (bigvgan.py:800-813, called through DotsModel._decode_latents,
 *     native/model.py:204-206, from DotsBatchEngine.vocode, engine.py:825-833);
 *   - strict streaming: AudioVAE.stream_step / stream_flush
 *     (bigvgan.py:1037-1050, native/model.py:208-218, engine.py:835-852):
 *     per chunk the LSTM front advances its state, the chunk joins a fixed
 *     window of frames, and the whole decoder re-runs over the window.
 * dvoc_decode is both, for many requests in one call: the front
 * (post_proj, Linear, LSTM, Linear; fp32), then the decoder (conv_pre, per
 * stage a causal transposed conv and the mean of its AMP resblocks of
 * anti-aliased SnakeBeta activations and causal dilated convs,
 * activation_post, conv_post, tanh) with every convolution on the tcgen05
 * tensor cores (fp16 operands: the 10-bit mantissa of tf32, the precision of
 * PyTorch's cuDNN convolutions on this GPU; fp32 accumulation) and everything
 * else in fp32.
 *
 * The same shared library (libdfm.so) exports these symbols next to the FM
 * head's (dfm.h); status codes and device error bits are dfm.h's.
 *
 * Conventions: as in dfm.h.  Every pointer inside the structs is a DEVICE
 * pointer; tensors are fp32 except the packed conv weights (fp16);
 * activations are frames-first ([request]
 * [frame][channel]); the caller owns every buffer.  The library owns only the
 * handle and its TMA descriptors; dvoc_decode allocates nothing and does not
 * synchronise.  Channel counts are padded to multiples of 32 inside the
 * library ("Cp" below: Cp(C) = 32 * ceil(C / 32)).
 */
#ifndef DVOC_H_
#define DVOC_H_

#include <stddef.h>
#include <stdint.h>

#include "dfm.h"

#ifdef __cplusplus
extern "C" {
#endif

#define DVOC_MAX_STAGES 8
#define DVOC_MAX_KERNELS 4

/* Decoder shape.  Mirrors the vocoder section of the checkpoint's config.json
 * (AudioVAEConfig, vocoder/config.py:6-24, read by Decoder.__init__,
 * bigvgan.py:542-612, and AudioVAE.__init__, bigvgan.py:751-788), restricted to
 * the causal decoder that strict streaming requires (bigvgan.py:937-940). */
typedef struct DvocConfig {
  int32_t latent_dim;                 /* L: latent channels */
  int32_t initial_channels;           /* upsample_initial_channel; stage i has initial/2^(i+1) channels */
  int32_t num_stages;                 /* len(upsample_rates), 1..DVOC_MAX_STAGES */
  int32_t upsample_rates[DVOC_MAX_STAGES];  /* u_i; the transposed conv of stage i has kernel 2 u_i */
  int32_t num_kernels;                /* resblocks per stage, 1..DVOC_MAX_KERNELS */
  int32_t resblock_kernel_sizes[DVOC_MAX_KERNELS];
  int32_t resblock_dilations[DVOC_MAX_KERNELS][3];
  int32_t resblock_type;              /* 1: AMPBlock1 (3 pairs of convs), 2: AMPBlock2 (2 convs) */
  int32_t mi_layers;                  /* LSTM layers of the front (mi_num_layers); hidden 4L */
  int32_t lookahead;                  /* num_decoder_lookahead: conv_pre has 2*lookahead+1 taps */
  int32_t use_tanh;                   /* use_tanh_at_final (else clamp to [-1, 1]) */
  int32_t max_batch;                  /* most requests one call carries */
  int32_t max_frames;                 /* most frames one call decodes (utterance or window) */
} DvocConfig;

/* Weights: the reference state dict (after remove_weight_norm), repacked by
 * nanovllm_dots_b200.vocoder.pack_voc_weights.  Front tensors keep the
 * reference layouts; the decoder's convolutions and activations are packed,
 * in execution order, as:
 *   conv_w: per conv [N][taps][Cp(Cin)] with N = Cp(Cout) (conv_pre and the
 *           resblock convs: W[co][ci][j] at [co][j][ci]) or u*Cp(Cout) (the
 *           transposed conv of a stage: tap 0 reads frame t-1 with
 *           W[ci][co][r+u], tap 1 frame t with W[ci][co][r], at row r*Cp(Cout)+co),
 *           as fp16 (round to nearest); order: conv_pre, then per stage its
 *           transposed conv and per resblock per layer convs1.l, convs2.l
 *           (type 1) or convs.l (type 2);
 *   conv_b: per conv [N] (a transposed conv's bias repeated per phase r);
 *   act:    per activation [Cp] exp(alpha), [Cp] 1/(exp(beta)+1e-9),
 *           [Cp][12] upsampling filter, [Cp][12] downsampling filter; order:
 *           per stage per resblock activations 0..5 (type 1) or 0..1 (type 2),
 *           then activation_post.  The resblock activations' filters are the
 *           reference's fixed buffers, the same for every channel: only
 *           channel 0's are read; activation_post's are per channel.
 * Padded channels hold zeros.  dvoc_conv_floats / dvoc_bias_floats /
 * dvoc_act_floats give the packed sizes. */
typedef struct DvocWeights {
  const float* post_w;      /* post_proj [L][L] (the 1x1 conv's weight[:, :, 0]) */
  const float* post_b;      /* [L] */
  const float* mi_in_w;     /* dec_mi_layer.0 [4L][L] */
  const float* mi_in_b;     /* [4L] */
  const float* lstm_w_ih;   /* [mi_layers][16L][4L], gate order i, f, g, o */
  const float* lstm_w_hh;   /* [mi_layers][16L][4L] */
  const float* lstm_b_ih;   /* [mi_layers][16L] */
  const float* lstm_b_hh;   /* [mi_layers][16L] */
  const float* mi_out_w;    /* dec_mi_layer.2 [L][4L] */
  const float* mi_out_b;    /* [L] */
  const void* conv_w;       /* packed decoder convs (above), fp16 */
  const float* conv_b;      /* packed decoder conv biases */
  const float* act;         /* packed alias-free activations */
  const float* post_conv_w; /* conv_post [7][Cp(C_last)]: weight[0][c][j] at [j][c] */
  const float* post_conv_b; /* [1], or NULL when use_bias_at_final is false */
} DvocWeights;

/* One call over n requests.
 *   One-shot (window == 0): request b's latents[b][0..lengths[b]) are decoded
 *     from a fresh LSTM state (lstm_h/lstm_c zero-filled by the caller) into
 *     audio[b][0 .. lengths[b]*hop); samples past that are unspecified.
 *     Replaces AudioVAE.inference_from_latents(do_sample=False) per request.
 *   Streaming (window > frames): each request's chunk of `frames` latent
 *     frames advances its LSTM state (lstm_h/lstm_c in and out) and is appended
 *     to its decoder window (windows[b], `valid[b]` frames valid before the
 *     call: min(total frames so far, window)); the decoder then runs over the
 *     whole window and audio[b] receives window*hop samples, of which the
 *     caller emits the stable ones (AudioVAE._slice_stream_audio_window,
 *     bigvgan.py:1005-1035).  Replaces AudioVAE.stream_step per request.
 *   Flush (window > 0, frames == 0): the decoder runs over the windows as
 *     they are (AudioVAE.stream_flush). */
typedef struct DvocBatch {
  int32_t n;                /* requests, 1..max_batch */
  int32_t frames;           /* latent frames per request in this call */
  int32_t window;           /* 0 (one-shot) or the stream window W (frames < W <= max_frames) */
  const float* latents;     /* [n][frames][L] (unused when frames == 0) */
  const int32_t* lengths;   /* one-shot: [n] valid frames (1..frames), or NULL for all */
  float* lstm_h;            /* [mi_layers][n][4L], in/out */
  float* lstm_c;            /* [mi_layers][n][4L], in/out */
  float* windows;           /* streaming: [n][window][L], in/out */
  const int32_t* valid;     /* streaming: [n] valid frames of each window before the call */
  float* audio;             /* [n][T*hop], T = window (streaming) or frames (one-shot) */
} DvocBatch;

/* Handle.  Validates the configuration (DFM_ERR_UNSUPPORTED outside the
 * supported family: causal decoder, latent_dim even and at most 192,
 * resblock type 1 or 2, every stage at least 1 channel) and encodes the
 * weights' TMA descriptors; copies no weights (they must outlive the handle).
 * conv_w, conv_b, act and lstm_w_hh must be 16-byte aligned.  A handle serves
 * one call at a time (it keeps the tensor maps of the last call's shape). */
int dvoc_create(const DvocConfig* cfg, const DvocWeights* w, void** handle);
int dvoc_destroy(void* handle);

/* Packed weight sizes in floats (0 for an invalid configuration). */
size_t dvoc_conv_floats(const DvocConfig* cfg);
size_t dvoc_bias_floats(const DvocConfig* cfg);
size_t dvoc_act_floats(const DvocConfig* cfg);

/* Audio samples per latent frame (the product of the upsample rates). */
int32_t dvoc_hop(const DvocConfig* cfg);

/* Frames of left context of strict streaming (Decoder._stream_left_context,
 * bigvgan.py:700-722); the stream window is chunk + lookahead + this. */
int32_t dvoc_stream_left_context(const DvocConfig* cfg);

/* Workspace bytes for calls up to max_batch x max_frames (256-byte aligned;
 * zero-filled once before first use). */
size_t dvoc_workspace_size(void* handle);

/* One call (see DvocBatch) on `stream`. */
int dvoc_decode(void* handle, const DvocBatch* batch, void* workspace, size_t workspace_bytes,
                void* stream);

/* Profiling: the number of decoder convolutions, and one of them (index in
 * execution order: conv_pre, then per stage its transposed conv and its
 * resblock convs) launched alone with the arguments a dvoc_decode of `batch`
 * would give it, reading whatever the workspace holds.  bench.py times the
 * decoder's own convolution launches with these; no reference counterpart. */
int32_t dvoc_num_convs(void* handle);
int dvoc_conv_launch(void* handle, const DvocBatch* batch, void* workspace, size_t workspace_bytes,
                     int32_t index, void* stream);

/* Synchronise `stream` and return the device error word of the workspace
 * (DFM_DEV_ERR_* bits: a bounded wait that gave up); the word is cleared. */
int dvoc_read_error(void* handle, void* workspace, void* stream, uint32_t* err_word);

#ifdef __cplusplus
}
#endif

#endif /* DVOC_H_ */
