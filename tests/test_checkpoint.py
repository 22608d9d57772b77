"""Checkpoint format version 1 (src/net/checkpoint/model.rs, io.rs) through
liboxf.so's C ABI, on the CPU: round trips, the fixtures in
tests/golden/checkpoint_v1 (reference serializer layout and an inline-table
layout), and every validation the reference performs on load."""
from __future__ import annotations

import re
import shutil
import tomllib
from pathlib import Path

import numpy as np
import pytest

from oxf import _lib, checkpoint as ck, models

GOLDEN = Path(__file__).resolve().parent / "golden" / "checkpoint_v1"


def _flat(n, seed=0):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


def _copy_fixture(tmp_path, name):
    for ext in (".toml", ".bin"):
        shutil.copy(GOLDEN / (name + ext), tmp_path / (name + ext))
    return tmp_path / (name + ".toml")


def _rewrite(path: Path, old: str, new: str) -> None:
    text = path.read_text()
    assert old in text, old
    path.write_text(text.replace(old, new, 1))


# ---------------------------------------------------------------- round trips
@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("act", [_lib.ACT_IDENTITY, _lib.ACT_GELU, _lib.ACT_RELU, _lib.ACT_SILU])
def test_linear_round_trip(tmp_path, bias, act):
    layer = models.Layer(5, 3, act, bias)
    flat = _flat(layer.count())
    ck.dump_linear(tmp_path / "lin", layer, flat)
    assert (tmp_path / "lin.toml").exists() and (tmp_path / "lin.bin").stat().st_size == 4 * flat.size
    got_layer, got = ck.load_linear(tmp_path / "lin")
    assert got_layer == layer
    np.testing.assert_array_equal(got, flat)


@pytest.mark.parametrize("res", [None, (0, 3), (1, 2)])
def test_mlp_round_trip(tmp_path, res):
    widths = [6, 12, 6, 6] if res != (1, 2) else [6, 12, 12, 4]
    layers = [models.Layer(widths[i], widths[i + 1], _lib.ACT_GELU if i == 0 else 0, i != 1)
              for i in range(3)]
    cfg = models.MlpConfig(layers, res)
    n = sum(l.count() for l in layers)
    flat = _flat(n, 1)
    ck.dump_mlp(tmp_path / "m.toml", cfg, flat)
    got_cfg, got = ck.load_mlp(tmp_path / "m.toml")
    assert got_cfg == cfg
    np.testing.assert_array_equal(got, flat)


@pytest.mark.parametrize("norm", [_lib.NORM_RMS, _lib.NORM_LAYER])
@pytest.mark.parametrize("bias", [False, True])
def test_transformer_round_trip(tmp_path, norm, bias):
    cfg = models.transformer_config(8, 16, 32, out=12, norm=norm, bias=bias)
    flat = models.init_transformer_params(cfg, seed=3)
    ck.dump_transformer_params(tmp_path / "model", cfg, flat)
    got_cfg, got = ck.load_transformer_params(tmp_path / "model")
    assert got_cfg == cfg
    np.testing.assert_array_equal(got, flat)


def test_written_metadata_follows_the_reference_schema(tmp_path):
    """Field names, types and contiguous cursor-order ranges of the written
    TOML, read back with an independent TOML parser (tomllib)."""
    cfg = models.transformer_config(8, 16, 32, bias=True)
    flat = models.init_transformer_params(cfg, seed=4)
    ck.dump_transformer_params(tmp_path / "model", cfg, flat)
    doc = tomllib.loads((tmp_path / "model.toml").read_text())
    assert {k: doc[k] for k in ("format_version", "model_type", "scalar_type", "data_file",
                                "data_bytes")} == {
        "format_version": 1, "model_type": "transformer", "scalar_type": "f32_le",
        "data_file": "model.bin", "data_bytes": 4 * flat.size}
    t = doc["transformer"]
    assert set(t) == {"block_count", "attention_residual", "feed_forward_residual",
                      "normalization", "position", "query", "key", "value", "feed_forward",
                      "output"}
    assert (t["block_count"], t["attention_residual"], t["feed_forward_residual"],
            t["normalization"]) == (1, True, True, "layer")
    assert set(t["query"]) == {"input_neurons", "output_neurons", "activation", "weights", "bias"}
    assert set(t["query"]["weights"]) == {"rows", "cols", "byte_start", "byte_end"}
    assert set(t["query"]["bias"]) == {"len", "byte_start", "byte_end"}
    ffn = t["feed_forward"]
    assert ffn["layer_count"] == 2 and ffn["loss"] == "mean_squared_error"
    assert "residual" not in ffn
    assert [l["activation"] for l in ffn["layers"]] == ["gelu", "identity"]
    # cursor order q, k, v, position, ffn layers, output; contiguous
    ranges = []
    for lin in (t["query"], t["key"], t["value"]):
        ranges += [lin["weights"], lin["bias"]]
    ranges.append(t["position"])
    for lin in ffn["layers"] + [t["output"]]:
        ranges += [lin["weights"], lin["bias"]]
    pos = 0
    for r in ranges:
        assert r["byte_start"] == pos
        n = r["rows"] * r["cols"] if "rows" in r else r["len"]
        pos = r["byte_end"]
        assert pos - r["byte_start"] == 4 * n
    assert pos == doc["data_bytes"]
    raw = np.fromfile(tmp_path / "model.bin", dtype="<f4")
    np.testing.assert_array_equal(raw, flat)


# ---------------------------------------------------------------- fixtures
def test_reads_reference_layout_fixtures():
    layer, lin = ck.load_linear(GOLDEN / "linear.toml")
    assert layer == models.Layer(4, 6, _lib.ACT_GELU, True)
    np.testing.assert_array_equal(lin, np.load(GOLDEN / "linear_params.npy"))
    cfg, mlp = ck.load_mlp(GOLDEN / "mlp")
    assert cfg == models.MlpConfig([models.Layer(4, 8, _lib.ACT_RELU, True),
                                    models.Layer(8, 4, _lib.ACT_IDENTITY, True)], (0, 2))
    np.testing.assert_array_equal(mlp, np.load(GOLDEN / "mlp_params.npy"))


def test_inline_table_layout_reads_the_same():
    a = ck.load_mlp(GOLDEN / "mlp.toml")
    b = ck.load_mlp(GOLDEN / "mlp_inline.toml")
    assert a[0] == b[0]
    np.testing.assert_array_equal(a[1], b[1])


def test_rewritten_fixture_is_byte_identical(tmp_path):
    """Our writer reproduces the reference serializer layout of the
    fixture (plain keys, [tables], [[layers]]) byte for byte."""
    cfg, flat = ck.load_mlp(GOLDEN / "mlp.toml")
    ck.dump_mlp(tmp_path / "mlp", cfg, flat)
    assert (tmp_path / "mlp.toml").read_text() == (GOLDEN / "mlp.toml").read_text()
    assert (tmp_path / "mlp.bin").read_bytes() == (GOLDEN / "mlp.bin").read_bytes()


# ---------------------------------------------------------------- paths (io.rs:14-50)
def test_path_rules(tmp_path):
    layer = models.Layer(2, 2)
    with pytest.raises(_lib.OxfError, match="must use .toml, not .json"):
        ck.dump_linear(tmp_path / "m.json", layer, _flat(4))
    ck.dump_linear(tmp_path / "m.v1.toml", layer, _flat(4))
    doc = tomllib.loads((tmp_path / "m.v1.toml").read_text())
    assert doc["data_file"] == "m.v1.bin" and (tmp_path / "m.v1.bin").exists()
    with pytest.raises(_lib.OxfError, match="must use .toml, not .bin"):
        ck.load_linear(tmp_path / "m.v1.bin")


def test_data_file_must_be_a_plain_name(tmp_path):
    p = _copy_fixture(tmp_path, "linear")
    _rewrite(p, 'data_file = "linear.bin"', 'data_file = "../linear.bin"')
    with pytest.raises(_lib.OxfError, match="plain file name"):
        ck.load_linear(p)


# ---------------------------------------------------------------- validation (model.rs:350-537)
@pytest.mark.parametrize("old,new,message", [
    ("format_version = 1", "format_version = 2", "unsupported checkpoint format version 2"),
    ('model_type = "linear"', 'model_type = "mlp"', 'model type "mlp", expected "linear"'),
    ('scalar_type = "f32_le"', 'scalar_type = "f64_le"', "unsupported scalar encoding"),
    ("data_bytes = 120", "data_bytes = 124", "ranges end at 120, metadata declares 124"),
    ("len = 6", "len = 5", "bias length does not match"),
    ("byte_start = 96", "byte_start = 100", "not the expected contiguous range"),
    ("rows = 4", "rows = 5", "weight shape does not match"),
    ("input_neurons = 4", "input_neurons = 0", "dimensions must be non-zero"),
    ('activation = "gelu"', 'activation = "tanh"', "unknown variant `tanh`"),
    ("input_neurons = 4\n", "", "missing field `input_neurons`"),
])
def test_linear_validation(tmp_path, old, new, message):
    p = _copy_fixture(tmp_path, "linear")
    _rewrite(p, old, new)
    with pytest.raises(_lib.OxfError, match=message):
        ck.load_linear(p)


def test_data_file_size_must_match(tmp_path):
    p = _copy_fixture(tmp_path, "linear")
    with open(tmp_path / "linear.bin", "ab") as f:
        f.write(b"\0\0\0\0")
    with pytest.raises(_lib.OxfError, match="data file has 124 bytes, metadata declares 120"):
        ck.load_linear(p)


@pytest.mark.parametrize("old,new,message", [
    ("layer_count = 2", "layer_count = 3", "layer_count is 3, but 2 layers"),
    ("start = 0\nend = 2", "start = 1\nend = 1", "invalid MLP residual range"),
    ("start = 0\nend = 2", "start = 0\nend = 1", "residual connects 4 input neurons to 8"),
    ('loss = "mean_squared_error"', 'loss = "cross_entropy"', "unknown variant `cross_entropy`"),
])
def test_mlp_validation(tmp_path, old, new, message):
    p = _copy_fixture(tmp_path, "mlp")
    _rewrite(p, old, new)
    with pytest.raises(_lib.OxfError, match=message):
        ck.load_mlp(p)


def test_mlp_connectivity(tmp_path):
    """Layer i must take what layer i-1 produces (model.rs:397-405)."""
    p = _copy_fixture(tmp_path, "mlp")
    text = p.read_text().replace("input_neurons = 8\n", "input_neurons = 6\n")
    text = text.replace("rows = 8\ncols = 4\nbyte_start = 160\nbyte_end = 288",
                        "rows = 6\ncols = 4\nbyte_start = 160\nbyte_end = 256")
    text = text.replace("byte_start = 288\nbyte_end = 304", "byte_start = 256\nbyte_end = 272")
    text = text.replace("data_bytes = 304", "data_bytes = 272")
    p.write_text(text)
    (tmp_path / "mlp.bin").write_bytes((tmp_path / "mlp.bin").read_bytes()[:272])
    with pytest.raises(_lib.OxfError, match="layer 1 expects 6 neurons, previous layer produces 8"):
        ck.load_mlp(p)


def _transformer_file(tmp_path, **kw):
    cfg = models.transformer_config(8, 16, 32, **kw)
    ck.dump_transformer_params(tmp_path / "t", cfg, models.init_transformer_params(cfg, seed=5))
    return tmp_path / "t.toml"


@pytest.mark.parametrize("old,new,message", [
    ("block_count = 1", "block_count = 2", "requires exactly one block"),
    ("attention_residual = true", "attention_residual = false", "requires both residual paths"),
    ('normalization = "layer"', 'normalization = "batch"', "unknown variant `batch`"),
])
def test_transformer_validation(tmp_path, old, new, message):
    p = _transformer_file(tmp_path)
    _rewrite(p, old, new)
    with pytest.raises(_lib.OxfError, match=message):
        ck.load_transformer_params(p)


def test_transformer_dimension_checks(tmp_path):
    """Q and K widths must match (model.rs:467-469): rewrite K's width
    consistently (shape, ranges, later offsets) so only that rule fails."""
    cfg = models.transformer_config(4, 8, 16)
    flat = models.init_transformer_params(cfg, seed=6)
    ck.dump_transformer_params(tmp_path / "t", cfg, flat)
    doc = tomllib.loads((tmp_path / "t.toml").read_text())
    k = doc["transformer"]["key"]
    assert k["output_neurons"] == 8
    head, sep, tail = (tmp_path / "t.toml").read_text().partition("[transformer.key]")
    tail = tail.replace("output_neurons = 8", "output_neurons = 4", 1)
    tail = tail.replace("rows = 8\ncols = 8", "rows = 8\ncols = 4", 1)
    # every later range shifts by the 32 removed floats (128 bytes)
    def shift(m):
        v = int(m.group(2))
        return f"{m.group(1)}{v - 128 if v > k['weights']['byte_start'] else v}"
    text = re.sub(r"(byte_(?:start|end) = )(\d+)", shift, head + sep + tail)
    text = text.replace(f"data_bytes = {4 * flat.size}", f"data_bytes = {4 * flat.size - 128}")
    (tmp_path / "t.toml").write_text(text)
    (tmp_path / "t.bin").write_bytes(np.zeros(flat.size - 32, "<f4").tobytes())
    with pytest.raises(_lib.OxfError, match="query and key dimensions must match"):
        ck.load_transformer_params(tmp_path / "t")


def test_parse_errors_are_reported(tmp_path):
    p = _copy_fixture(tmp_path, "linear")
    _rewrite(p, "rows = 4", "rows = 4.0")
    with pytest.raises(_lib.OxfError, match="TOML parse error at line"):
        ck.load_linear(p)


# ---------------------------------------------------------------- property tests
from hypothesis import HealthCheck, given, settings, strategies as st  # noqa: E402

ACTS = [_lib.ACT_IDENTITY, _lib.ACT_GELU, _lib.ACT_RELU, _lib.ACT_SILU]
PROPERTY = settings(max_examples=40, deadline=None,
                    suppress_health_check=[HealthCheck.function_scoped_fixture])


@st.composite
def mlp_configs(draw):
    """Any MLP the format describes: 1-6 connected Linear layers of widths
    1-9, any activation, bias or not, and optionally a residual range
    [start, end) whose input and output widths agree."""
    n = draw(st.integers(1, 6))
    widths = draw(st.lists(st.integers(1, 9), min_size=n + 1, max_size=n + 1))
    acts = draw(st.lists(st.sampled_from(ACTS), min_size=n, max_size=n))
    bias = draw(st.lists(st.booleans(), min_size=n, max_size=n))
    res = None
    if draw(st.booleans()):
        start = draw(st.integers(0, n - 1))
        end = draw(st.integers(start + 1, n))
        widths[end] = widths[start]
        res = (start, end)
    layers = [models.Layer(widths[i], widths[i + 1], acts[i], bias[i]) for i in range(n)]
    return models.MlpConfig(layers, res)


@PROPERTY
@given(cfg=mlp_configs(), seed=st.integers(0, 2**31 - 1))
def test_mlp_round_trip_any_spec(tmp_path, cfg, seed):
    flat = _flat(sum(l.count() for l in cfg.layers), seed)
    ck.dump_mlp(tmp_path / "any.toml", cfg, flat)
    assert (tmp_path / "any.bin").stat().st_size == 4 * flat.size
    got_cfg, got = ck.load_mlp(tmp_path / "any.toml")
    assert got_cfg == cfg
    np.testing.assert_array_equal(got, flat)


@PROPERTY
@given(seq=st.integers(1, 6), hidden=st.integers(1, 8), ffn=st.integers(1, 10),
       out=st.integers(1, 7), norm=st.sampled_from([_lib.NORM_RMS, _lib.NORM_LAYER]),
       bias=st.booleans(), seed=st.integers(0, 2**31 - 1))
def test_transformer_round_trip_any_dims(tmp_path, seq, hidden, ffn, out, norm, bias, seed):
    cfg = models.transformer_config(seq, hidden, ffn, out=out, norm=norm, bias=bias)
    flat = _flat(cfg.param_count(), seed)
    ck.dump_transformer_params(tmp_path / "anyt", cfg, flat)
    got_cfg, got = ck.load_transformer_params(tmp_path / "anyt")
    assert got_cfg == cfg
    np.testing.assert_array_equal(got, flat)
