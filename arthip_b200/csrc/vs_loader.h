// The VapourSynth filter's loading path and frame IO, in the engine core (no VapourSynth
// or protobuf headers): the fp32 -> fp16 model conversion, loadONNX's input-shape fixing,
// the hip.Model argument / clip-format validation, and the packing of clip planes into the
// engine's NCHW host buffer and back. A thin plugin shim maps VapourSynth's API onto
// these (ah_vs_* in include/arthip_b200.h).
//
// Follows src/vapoursynth/convert_float_to_float16.cpp:165-186,294-611 (itself a restatement
// of onnxruntime's python/tools/transformers/float16.py, v1.10.0),
// src/vapoursynth/onnx_utils.cpp:29-128 and src/vapoursynth/vs_hip.cpp:77-591.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_set>

#include "onnx_wire.h"

namespace ah {
namespace vs {

// ---------------------------------------------------------------------------
// fp32 -> fp16 model conversion
// ---------------------------------------------------------------------------
struct Fp16Options {
  bool force_fp16_initializers = true;
  std::unordered_set<std::string> op_block_list;  // op types kept in fp32 (Casts inserted around them)
  bool cast_input = false;   // keep fp32 graph inputs: insert an fp32 -> fp16 Cast after each
  bool cast_output = false;  // keep fp32 graph outputs: insert an fp16 -> fp32 Cast before each
};

// Converts `m` in place: fp32 initializers become fp16 with the converter's own rounding
// (round to nearest even, results below the fp16 normal range flushed to signed zero,
// overflow and NaN to signed infinity), fp32 graph inputs / outputs become fp16 unless cast
// (then a boundary Cast named graph_input_cast_<i> / graph_output_cast_<i> is inserted),
// Cast-to-fp32 nodes become Cast-to-fp16, and nodes of blocked op types get Casts around
// their fp16 inputs and outputs. `note` receives a warning when an initializer is used by
// both blocked and converted nodes.
void ConvertFloatToFloat16(onnx::Model* m, const Fp16Options& opt, std::string* note);

// loadONNX's specifyShape: exactly one graph input and one output, both rank 4; the input
// gets batch N, height tile_h and width tile_w (0 keeps 0, as the reference passes), the
// output batch N and unknown height / width. Returns false with a message.
bool SpecifyShape(onnx::Model* m, int64_t tile_w, int64_t tile_h, int64_t batch, std::string* err);

// ---------------------------------------------------------------------------
// hip.Model arguments and clip formats (VapourSynth's VSColorFamily / VSSampleType values)
// ---------------------------------------------------------------------------
enum ColorFamily : int { kCfUndefined = 0, kCfGray = 1, kCfRGB = 2, kCfYUV = 3 };
enum SampleType : int { kStInteger = 0, kStFloat = 1 };

struct ClipFormat {
  int color_family = kCfUndefined;
  int sample_type = kStInteger;
  int bits_per_sample = 8;
  int subsampling_w = 0, subsampling_h = 0;
  int num_planes = 1;
  int width = 0, height = 0;
};

struct ModelArgs {
  int device_id = 0;
  int num_streams = 1;
  int overlap_n = 0;
  int64_t overlap[2] = {0, 0};
  int tilesize_n = 0;
  int64_t tilesize[2] = {0, 0};
};

// Static clip checks at creation (vs_hip.cpp:372-393): family, sample type / depth,
// subsampling. Empty string when accepted.
std::string ValidateClipFormat(const ClipFormat& f);
// overlap / tilesize: only the no-tiling default is accepted (vs_hip.cpp:414-442).
std::string ValidateTiling(const ModelArgs& a, const ClipFormat& clip);
// Plane count against the model's input channels (vs_hip.cpp:487-497).
std::string ValidateChannels(const ClipFormat& f, int model_in_channels);

// Packs `planes` (one pointer and byte stride per plane, every plane width x height) into
// a plane-major NCHW buffer: fp32 when `to_fp32`, else fp16 bits (round to nearest even).
// Integer samples are scaled to [0, 1] (8-bit / 255, 16-bit / 65535); fp16 samples are
// copied or widened; fp32 samples converted or copied (vs_hip.cpp:160-243).
void PackPlanes(const ClipFormat& f, const void* const* planes, const ptrdiff_t* strides, bool to_fp32,
                void* dst);
// Writes output channel c of the engine's NCHW result (out_w x out_h per channel, fp32 or
// fp16 bits) into dst_planes[c] for c < n_planes: as fp32, as fp16, or as 16-bit integers
// (v * 65535 + 0.5, clamped to [0, 65535] and truncated) when `as_int16` (vs_hip.cpp:257-435).
void UnpackPlanes(const void* src, bool src_fp32, int out_w, int out_h, void* const* dst_planes,
                  const ptrdiff_t* dst_strides, int n_planes, bool as_int16);

}  // namespace vs
}  // namespace ah
