"""CPU tests of the host side of libq8cuda: the shared library loads and exports
every symbol the C header declares, the tensor-parallel shard plan, the
safetensors scanner (including failure modes), RoPE frequencies, configs.
No kernel is launched."""
import json
import os
import re
import struct

import numpy as np
import pytest

from lama32_mojo_b200 import PRESETS, _lib
from lama32_mojo_b200 import config as cfgmod
from lama32_mojo_b200 import model as M
from oracle import q8_oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    txt = open(os.path.join(REPO, "include", "q8cuda.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(q8(?:op)?_[a-z0-9_]+)\s*\(", txt)))


def test_library_loads_and_exports_header_symbols():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # every declared function has a ctypes signature
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)
    assert b"sm_100a" in L.q8_version()
    assert L.q8_status_string(_lib.Q8_ERR_KV_FULL) == b"KV cache full"


def test_status_codes_match_header():
    txt = open(os.path.join(REPO, "include", "q8cuda.h")).read()
    for name in ("Q8_OK", "Q8_ERR_ARG", "Q8_ERR_CUDA", "Q8_ERR_OOM", "Q8_ERR_KV_FULL", "Q8_ERR_IO",
                 "Q8_ERR_FORMAT", "Q8_ERR_COMM", "Q8_ERR_TIMEOUT", "Q8_ERR_STATE"):
        v = int(re.search(name + r"\s*=\s*(\d+)", txt).group(1))
        assert getattr(_lib, name) == v


def test_config_struct_layout():
    import ctypes as C
    # int32 x7 + float (32 B), double x5 (40 B), int32 x4 (16 B) on x86-64
    assert C.sizeof(_lib.q8_config) == 88
    assert _lib.q8_config.theta.offset == 32 and _lib.q8_config.rope_type.offset == 72
    assert _lib.q8_config.weight_dtype.offset == 84


def test_config_weight_dtype_to_c():
    """The bf16 shells' configs select bf16 weights; everything else packed Q8."""
    from lama32_mojo_b200 import PRESETS
    cfg = PRESETS["tiny-llama"]
    assert cfg.to_c().weight_dtype == _lib.Q8_PACKED
    assert cfg.replace(weights="bf16").to_c().weight_dtype == _lib.Q8_BF16
    # decode bytes count 2-byte weights for bf16, 33/32 bytes for Q8
    w8 = cfg.decode_bytes(1, 0)
    w16 = cfg.replace(weights="bf16").decode_bytes(1, 0)
    assert abs(w16 / w8 - 2.0 / (1 + 2 / 64)) < 1e-9


@pytest.mark.parametrize("name", ["llama-3.2-1b", "llama-3.1-8b", "qwen3-8b", "tiny-llama"])
def test_rope_inv_freq_matches_oracle(name):
    import ctypes as C
    cfg = PRESETS[name]
    out = np.zeros(cfg.head_dim // 2, np.float32)
    c = cfg.to_c()
    _lib.check(_lib.lib().q8_rope_inv_freq(C.byref(c), out.ctypes.data_as(C.c_void_p)))
    ref = O.inv_freq(O.PRESETS[name])
    ulp = np.abs(out.view(np.int32).astype(np.int64) - ref.view(np.int32).astype(np.int64))
    assert ulp.max() <= 1


def test_presets_agree_with_oracle():
    for k, c in PRESETS.items():
        o = O.PRESETS[k]
        for f in ("hidden", "layers", "n_heads", "n_kv", "head_dim", "inter", "vocab", "eps", "theta",
                  "rope_type", "rope_factor", "qk_norm", "tied"):
            assert getattr(c, f) == getattr(o, f), (k, f)
        assert c.weight_names() == O.weight_names(o)


def test_config_from_reference_style_hf_json(tmp_path):
    j = {"hidden_size": 2048, "num_hidden_layers": 16, "num_attention_heads": 32, "num_key_value_heads": 8,
         "head_dim": 64, "intermediate_size": 8192, "vocab_size": 128256, "rms_norm_eps": 1e-5,
         "rope_theta": 500000.0, "tie_word_embeddings": True, "model_type": "llama",
         "rope_scaling": {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
                          "original_max_position_embeddings": 8192, "rope_type": "llama3"}}
    p = tmp_path / "config.json"
    p.write_text(json.dumps(j))
    c = cfgmod.from_hf_config(str(p))
    ref = PRESETS["llama-3.2-1b"]
    for f in ("hidden", "layers", "n_heads", "n_kv", "head_dim", "inter", "vocab", "eps", "theta", "rope_type",
              "rope_factor", "tied", "qk_norm"):
        assert getattr(c, f) == getattr(ref, f), f


@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_shard_plan_partitions_every_tensor(tp):
    """Concatenating the shards of every rank reproduces each tensor exactly once."""
    cfg = PRESETS["llama-3.1-8b"].replace(layers=1)
    for name in cfg.weight_names():
        shp = cfg.tensor_shape(name)
        plans = [M.shard_plan(cfg, r, tp, name) for r in range(tp)]
        assert all(p["n"] == shp[0] for p in plans)
        if len(shp) == 1:
            assert all(p["m"] == 1 and p["nrows"] == shp[0] for p in plans)
            continue
        kinds = {(p["nrows"] == shp[0], p["kl"] == shp[1]) for p in plans}
        if tp == 1:
            assert kinds == {(True, True)}
            continue
        if all(p["kl"] == shp[1] for p in plans) and all(p["nrows"] == shp[0] for p in plans):
            assert name == "model.embed_tokens.weight"  # replicated
            continue
        if all(p["kl"] == shp[1] for p in plans):  # row split
            rows = sorted((p["row0"], p["row0"] + p["nrows"]) for p in plans)
            assert rows[0][0] == 0 and rows[-1][1] == shp[0]
            assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
        else:  # K split
            ks = sorted((p["k0"], p["k0"] + p["kl"]) for p in plans)
            assert ks[0][0] == 0 and ks[-1][1] == shp[1] and all(a[1] == b[0] for a, b in zip(ks, ks[1:]))
            assert all(p["kl"] % 64 == 0 for p in plans)


def test_shard_plan_tied_head_not_loaded():
    cfg = PRESETS["llama-3.2-1b"]
    assert M.shard_plan(cfg, 0, 1, "lm_head.weight")["slot"] == ""
    assert M.shard_plan(cfg, 0, 1, "model.rotary_emb.inv_freq")["slot"] == ""


# ---------------------------------------------------------------- safetensors scanner
def write_st(path, tensors, meta=None):
    """Tiny safetensors writer: tensors = {name: (dtype_str, shape, bytes)}."""
    hdr, blobs, off = {}, [], 0
    if meta:
        hdr["__metadata__"] = meta
    for k, (dt, shp, b) in tensors.items():
        hdr[k] = {"dtype": dt, "shape": list(shp), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def test_inspect_single_and_sharded(tmp_path):
    a = np.arange(6, dtype=np.uint16).tobytes()
    write_st(tmp_path / "model.safetensors", {"x": ("BF16", (2, 3), a), "y": ("F16", (3,), a[:6])},
             meta={"format": "pt"})
    t = {r[0]: r for r in M.inspect_checkpoint(str(tmp_path))}
    assert set(t) == {"x", "y"} and t["x"][1] == "BF16" and t["x"][2] == (2, 3)
    assert t["x"][4] - t["x"][3] == 12
    d = tmp_path / "sh"
    d.mkdir()
    write_st(d / "a.safetensors", {"p": ("BF16", (4,), b"\0" * 8)})
    write_st(d / "b.safetensors", {"q": ("BF16", (2,), b"\0" * 4)})
    (d / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"p": "a.safetensors",
                                                                              "q": "b.safetensors"}}))
    names = {r[0]: r for r in M.inspect_checkpoint(str(d))}
    assert set(names) == {"p", "q"} and names["q"][1] == "BF16"


def test_inspect_rejects_truncated_and_corrupt(tmp_path):
    write_st(tmp_path / "model.safetensors", {"x": ("BF16", (64, 64), b"\0" * 8192)})
    raw = (tmp_path / "model.safetensors").read_bytes()
    (tmp_path / "model.safetensors").write_bytes(raw[:-100])
    with pytest.raises(_lib.Q8Error) as e:
        M.inspect_checkpoint(str(tmp_path))
    assert e.value.status == _lib.Q8_ERR_FORMAT and "truncated" in str(e.value)
    (tmp_path / "model.safetensors").write_bytes(struct.pack("<Q", 20) + b'{"x": {"dtype": 3,,}')
    with pytest.raises(_lib.Q8Error):
        M.inspect_checkpoint(str(tmp_path))
    (tmp_path / "model.safetensors").write_bytes(struct.pack("<Q", 1 << 40))
    with pytest.raises(_lib.Q8Error):
        M.inspect_checkpoint(str(tmp_path))
    with pytest.raises(_lib.Q8Error):
        M.inspect_checkpoint(str(tmp_path / "nope"))


class _StubModel:
    """Stands in for the device model behind Q8Model.chat_generate: a fixed
    token script, a KV counter and the sampling settings it was given."""

    def __init__(self, script, maxlen):
        self.script, self.maxlen, self.n, self.calls, self.sampling = list(script), maxlen, 0, [], None

    def set_sampling(self, temp, top_p, seed):
        self.sampling = (temp, top_p, seed)

    def forward_argmax(self, ids, seq=0):
        self.calls.append(list(ids))
        self.n += len(ids)
        return self.script[len(self.calls) - 1]

    def get_n_cached(self, seq=0):
        return self.n


def _chat(stub, ids, **kw):
    return M.Q8Model.chat_generate(stub, ids, **kw)


def test_chat_generate_control_flow():
    """The REPL loop of chat_q8.mojo:53-97: stop before EOS, stop at a full
    context, feed each token back, pass the sampling settings through."""
    s = _StubModel([7, 8, 9, 2, 5, 6], maxlen=100)
    assert _chat(s, [1, 2, 3], temp=0.6, top_p=0.9, eos=2, seed=4) == [7, 8, 9]
    assert s.calls == [[1, 2, 3], [7], [8], [9]] and s.sampling == (0.6, 0.9, 4)
    s = _StubModel([7, 8, 9, 10, 11, 12, 13], maxlen=6)  # 3 prompt tokens + 3 steps fill it
    assert _chat(s, [1, 2, 3]) == [7, 8, 9] and s.n == 6
    s = _StubModel([7, 8, 9, 10, 11], maxlen=100)
    assert _chat(s, [1], max_new=2) == [7, 8]
    s = _StubModel([2], maxlen=100)
    assert _chat(s, [1], eos=2) == []


def test_sample_draw_is_uniform_24_bit():
    """The model's per-row draws: 24-bit values in [0, 1), reproducible, and
    different for neighbouring sequences and positions."""
    d = [M.sample_draw(5, s, p) for s in range(4) for p in range(256)]
    assert all(0.0 <= v < 1.0 and float(v) * 2 ** 24 == int(float(v) * 2 ** 24) for v in d)
    assert len(set(d)) == len(d)
    assert M.sample_draw(5, 1, 7) == M.sample_draw(5, 1, 7) != M.sample_draw(6, 1, 7)
    assert 0.4 < float(np.mean(d)) < 0.6
