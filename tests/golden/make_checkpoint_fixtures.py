"""Writes the checkpoint-v1 fixtures in tests/golden/checkpoint_v1/.

The metadata files are written out here as text, laid out the way the
reference's serializer writes its structs (src/net/checkpoint/io.rs:52-58
uses toml::to_string_pretty on the structs of model.rs:23-51, linear.rs:
79-86, mlp.rs:21-34, metadata.rs:5-19): plain keys, then one [table] per
nested struct, one [[array]] entry per MLP layer. mlp_inline.toml holds the
same model with inline tables, comments and reordered keys, which a TOML
reader must accept alike. Parameters are seeded normals, little-endian f32.

    python tests/golden/make_checkpoint_fixtures.py
"""
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "checkpoint_v1"

LINEAR_TOML = """format_version = 1
model_type = "linear"
scalar_type = "f32_le"
data_file = "linear.bin"
data_bytes = 120

[linear]
input_neurons = 4
output_neurons = 6
activation = "gelu"

[linear.weights]
rows = 4
cols = 6
byte_start = 0
byte_end = 96

[linear.bias]
len = 6
byte_start = 96
byte_end = 120
"""

MLP_TOML = """format_version = 1
model_type = "mlp"
scalar_type = "f32_le"
data_file = "mlp.bin"
data_bytes = 304

[mlp]
layer_count = 2
loss = "mean_squared_error"

[mlp.residual]
start = 0
end = 2

[[mlp.layers]]
input_neurons = 4
output_neurons = 8
activation = "relu"

[mlp.layers.weights]
rows = 4
cols = 8
byte_start = 0
byte_end = 128

[mlp.layers.bias]
len = 8
byte_start = 128
byte_end = 160

[[mlp.layers]]
input_neurons = 8
output_neurons = 4
activation = "identity"

[mlp.layers.weights]
rows = 8
cols = 4
byte_start = 160
byte_end = 288

[mlp.layers.bias]
len = 4
byte_start = 288
byte_end = 304
"""

MLP_INLINE_TOML = """# the same MLP, written with inline tables
data_bytes = 304
format_version = 1
scalar_type = 'f32_le'
model_type = "mlp"
data_file = "mlp_inline.bin"

[mlp]
loss = "mean_squared_error"   # the only loss of version 1
layer_count = 2
residual = { start = 0, end = 2 }
layers = [
  { input_neurons = 4, output_neurons = 8, activation = "relu",
    weights = { rows = 4, cols = 8, byte_start = 0, byte_end = 128 },
    bias = { len = 8, byte_start = 128, byte_end = 160 } },
  { input_neurons = 8, output_neurons = 4, activation = "identity",
    weights = { rows = 8, cols = 4, byte_start = 160, byte_end = 288 },
    bias.len = 4, bias.byte_start = 288, bias.byte_end = 304 },
]
"""


def main() -> None:
    OUT.mkdir(exist_ok=True)
    rng = np.random.default_rng(20260101)
    lin = rng.standard_normal(4 * 6 + 6).astype("<f4")
    mlp = rng.standard_normal(4 * 8 + 8 + 8 * 4 + 4).astype("<f4")
    (OUT / "linear.toml").write_text(LINEAR_TOML)
    lin.tofile(OUT / "linear.bin")
    np.save(OUT / "linear_params.npy", lin.astype(np.float32))
    (OUT / "mlp.toml").write_text(MLP_TOML)
    mlp.tofile(OUT / "mlp.bin")
    (OUT / "mlp_inline.toml").write_text(MLP_INLINE_TOML)
    mlp.tofile(OUT / "mlp_inline.bin")
    np.save(OUT / "mlp_params.npy", mlp.astype(np.float32))


if __name__ == "__main__":
    main()
