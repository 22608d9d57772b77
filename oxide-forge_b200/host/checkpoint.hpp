// checkpoint.hpp — the reference's checkpoint format, version 1
// (src/net/checkpoint/model.rs, io.rs; src/net/metadata.rs): a TOML
// metadata file with parameter byte ranges, next to a binary file of
// little-endian f32 parameters in cursor order.
#pragma once
#include <cstddef>
#include <string>
#include <vector>

#include "oxf_host.h"

namespace oxf::ckpt {

enum class ModelType { Linear, Mlp, Transformer };

// A model read from (or to be written to) a checkpoint, in this library's
// spec types, with its parameters in cursor order (per Linear: weights
// [in, out] row-major then bias; transformer: q, k, v, position, the
// feed-forward layers, output).
struct Model {
  ModelType type = ModelType::Linear;
  oxf_layer_spec linear{};
  oxf_mlp_spec mlp{};
  oxf_transformer_spec transformer{};
  std::vector<float> params;
};

// Parameter count of a spec (what the .bin holds, divided by 4).
size_t param_count(const oxf_layer_spec& s);
size_t param_count(const oxf_mlp_spec& s);
size_t param_count(const oxf_transformer_spec& s);

// dump_* (model.rs:53-71, 209-247): writes <path>.toml and <path>.bin.
// Throws oxf::Error on a bad path, a spec the format cannot describe, a
// parameter count that does not match the spec, or an I/O failure.
void write(const std::string& path, const Model& model);

// load_* (model.rs:73-208, 249-298): reads and validates the metadata
// (format version, model type, scalar encoding, contiguous byte ranges,
// shapes, Linear connectivity, residual and transformer dimensions) and
// the data file size, then reads the parameters.
Model read(const std::string& path, ModelType expected);

}  // namespace oxf::ckpt
