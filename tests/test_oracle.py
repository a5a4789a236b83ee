"""The CPU oracle against the golden vectors made by the reference's own Python
(tests/golden/make_golden.py): pack_q8 bit-exactness, the seeded synthetic
checkpoints, prefill outputs of the three gen_oracle scripts and the cached
decode of bench_python.  CPU only."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import q8_oracle as O


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_pack_cases_bit_exact(golden_dir):
    pc = _load(golden_dir, "pack_cases.npz")
    n = 0
    for k in pc.files:
        if k.endswith("_in"):
            got = O.pack_q8(pc[k])
            exp = pc[k[:-3] + "_out"]
            assert got.dtype == np.uint16 and got.shape == exp.shape, k
            assert np.array_equal(got, exp), f"{k}: {(got != exp).sum()} u16 differ"
            n += 1
    assert n >= 5


def test_pack_layout_and_edge_semantics():
    # zero group -> scale 0, codes 0; underflowing scale -> +-127 for nonzero values
    w = np.zeros((2, 64), np.float32)
    w[1, :3] = [1e-7, -2e-6, 0.0]
    p = O.pack_q8(O.bf16_round(w))
    assert p.shape == (2, O.q8_rowstride(64))
    s, q = O.unpack_q8(p, 64)
    assert (s.view(np.uint16) == 0).all()
    assert q[1, :3].tolist() == [127, -127, 0] and (q[0] == 0).all()
    # codes never reach -128
    r = np.random.default_rng(0).standard_normal((16, 512)).astype(np.float32)
    _, q = O.unpack_q8(O.pack_q8(O.bf16_round(r)), 512)
    assert q.min() >= -127 and q.max() <= 127 and np.abs(q).max() == 127


def test_checkpoint_shas(golden_dir):
    man = json.load(open(os.path.join(golden_dir, "manifest.json")))
    for name, shas in man["checkpoints"].items():
        if name not in ("tiny-llama", "tiny-llama-untied", "tiny-qwen3"):
            continue  # the full-size sha list is checked on the GPU against the GPU packer
        ck = O.make_q8_checkpoint(O.PRESETS[name])
        assert set(ck) == set(shas)
        for t, want in shas.items():
            assert hashlib.sha256(np.ascontiguousarray(ck[t]).tobytes()).hexdigest() == want, (name, t)


@pytest.mark.parametrize("fixture,cfgname", [("tiny_llama_prefill.npz", "tiny-llama"),
                                             ("tiny_llama_untied_prefill.npz", "tiny-llama-untied"),
                                             ("tiny_qwen3_prefill.npz", "tiny-qwen3")])
def test_prefill_matches_reference_gen_oracle(golden_dir, fixture, cfgname):
    g = _load(golden_dir, fixture)
    cfg = O.PRESETS[cfgname]
    m = O.OracleModel(cfg, O.make_q8_checkpoint(cfg))
    lg = m.forward(list(g["ids"]))
    for L in (0, 1):
        np.testing.assert_allclose(m.trace[f"after_layer{L}"], g[f"after_layer{L}"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(lg, g["last_logits"], rtol=0, atol=1e-6)


def test_cached_decode_matches_reference_bench_python(golden_dir):
    g = _load(golden_dir, "tiny_qwen3_decode.npz")
    cfg = O.PRESETS["tiny-qwen3"]
    m = O.OracleModel(cfg, O.make_q8_checkpoint(cfg))
    lg = [m.forward(list(g["ids"]))]
    for t in g["tokens"][:-1]:
        lg.append(m.forward([int(t)]))
    lg = np.stack(lg)
    assert O.rel_l2(lg, g["logits"]) < 1e-5
    assert [int(np.argmax(x)) for x in lg] == g["tokens"].tolist()


def test_config0_fixture_consistent(golden_dir):
    path = os.path.join(golden_dir, "config0_llama1b.npz")
    if not os.path.exists(path):
        pytest.skip("config0 fixture not generated")
    g = np.load(path)
    # oracle prefill logits (committed) equal the reference gen_oracle logits
    np.testing.assert_allclose(g["oracle_prefill_logits"], g["last_logits"], rtol=0, atol=1e-5)
    assert g["tokens"].shape == (33,) and g["ids"].shape == (16,)
    assert int(np.argmax(g["last_logits"])) == int(g["tokens"][0])


def test_oracle_incremental_equals_prefill():
    """Size-independent property: prefill of s tokens == s cached single-token steps."""
    cfg = O.PRESETS["tiny-llama-untied"]
    ck = O.make_q8_checkpoint(cfg)
    ids = O.random_ids(cfg, 6, seed=5)
    a = O.OracleModel(cfg, ck)
    la = a.forward(ids)
    b = O.OracleModel(cfg, ck)
    for t in ids:
        lb = b.forward([t])
    assert O.rel_l2(lb, la) < 1e-5


def test_mm_q8_equals_dequant_matmul():
    rng = np.random.default_rng(3)
    w = O.pack_q8(O.bf16_round(rng.standard_normal((40, 256), dtype=np.float32) * 0.02))
    x = rng.standard_normal((3, 256), dtype=np.float32)
    y1 = O.mm_q8(x, w, 256)
    y2 = x @ O.dequant_q8(w, 256).T
    assert O.rel_l2(y1, y2) < 1e-6


def test_kv_full_raises():
    cfg = O.PRESETS["tiny-qwen3"]
    m = O.OracleModel(cfg, O.make_q8_checkpoint(cfg), maxlen=4)
    m.forward([1, 2, 3])
    with pytest.raises(RuntimeError, match="KV cache full"):
        m.forward([4, 5])


def _sample_rows(seed):
    """Logit rows for the sampler checks: continuous values, planted equal
    values (ties, a shared maximum), and rows with few distinct values."""
    rng = np.random.default_rng(seed)
    rows = []
    for n, scale in ((50, 3.0), (300, 1.0), (300, 8.0)):
        rows.append((rng.standard_normal(n) * scale).astype(np.float32))
    x = (rng.standard_normal(200) * 2).astype(np.float32)
    x[[5, 17, 90]] = x.max()  # three equal maxima
    x[[30, 31, 150, 199]] = x[40]
    rows.append(x)
    rows.append(rng.integers(-3, 1, 240).astype(np.float32) * np.float32(0.5))  # 4 values, big tie groups
    return rows


def test_sample_c_restatement_matches_literal():
    """The C restatement of sample() (oracle/q8_ref.c, the GPU checker)
    agrees with the loop-for-loop Python one on rows with and without ties;
    a disagreement is only tolerated where one ulp of exp() could flip the
    decision (margin)."""
    from oracle import q8_ref as R
    rng = np.random.default_rng(5)
    checked = 0
    for x in _sample_rows(3):
        for temp in (0.0, -1.0, 0.7, 1.0, 1.8):
            for top_p in (0.25, 0.9, 1.0):
                for u in (0.0, float(rng.random()), float(rng.random()), 0.9999999):
                    want = O.sample_literal(x, temp, top_p, u)
                    got, margin = R.sample(x, temp, top_p, u)
                    assert got == want or margin < 1e-6, (temp, top_p, u, got, want, margin)
                    checked += got == want
    assert checked > 0.99 * 5 * 5 * 3 * 4


@pytest.mark.parametrize("cfgname", ["tiny-llama", "tiny-qwen3", "tiny-llama-untied"])
def test_c_whole_model_matches_pinned_oracle(cfgname):
    """The C restatement's whole-model loop (oracle.q8_ref.RefModel, the
    checker of the full-size GPU parity tests) against the numpy oracle,
    which is pinned to the reference's own gen_oracle / bench_python output:
    per-layer residuals, last logits and greedy tokens of a cached decode."""
    from oracle import q8_ref as R
    cfg = O.PRESETS[cfgname]
    ck = O.make_q8_checkpoint(cfg)
    ids = O.random_ids(cfg, 13, seed=5)
    orc = O.OracleModel(cfg, ck)
    ref_lg = orc.forward(ids)
    ref_h = {i: orc.trace[f"after_layer{i}"] for i in (0, 1)}
    rm = R.RefModel(cfg, ck, O.inv_freq(cfg), maxlen=32)
    lg, hid = rm.prefill(ids, keep=(0, 1))
    for i in (0, 1):
        assert O.rel_l2(hid[i], ref_h[i]) < 1e-5
    assert O.rel_l2(lg, ref_lg) < 1e-5 and np.abs(lg - ref_lg).max() < 1e-4
    t_ref, t_c = int(np.argmax(ref_lg)), int(np.argmax(lg))
    assert t_ref == t_c
    for _ in range(4):
        t_ref = orc.forward_argmax([t_ref])
        t_c = int(np.argmax(rm.token(t_c)))
        assert t_ref == t_c


def test_bf16_prefill_matches_reference_gen_oracle(golden_dir):
    """bf16 weights (the non-Q8 path): gen_oracle.layer over the checkpoint
    widened to f32, norm weights 1 + N(0, 0.1)."""
    g = _load(golden_dir, "tiny_llama_bf16_prefill.npz")
    cfg = O.PRESETS["tiny-llama"].replace(weights="bf16")
    m = O.OracleModel(cfg, O.make_bf16_checkpoint(cfg, seed=5, norm_std=0.1))
    lg = m.forward(list(g["ids"]))
    for L in (0, 1):
        np.testing.assert_allclose(m.trace[f"after_layer{L}"], g[f"after_layer{L}"], rtol=0, atol=1e-6)
    np.testing.assert_allclose(lg, g["last_logits"], rtol=0, atol=1e-6)


def test_bf16_cached_decode_matches_reference_bench_python(golden_dir):
    g = _load(golden_dir, "tiny_qwen3_bf16_decode.npz")
    cfg = O.PRESETS["tiny-qwen3"].replace(weights="bf16")
    m = O.OracleModel(cfg, O.make_bf16_checkpoint(cfg, seed=6, norm_std=0.1))
    lg = [m.forward(list(g["ids"]))]
    for t in g["tokens"][:-1]:
        lg.append(m.forward([int(t)]))
    lg = np.stack(lg)
    assert O.rel_l2(lg, g["logits"]) < 1e-5
    assert [int(np.argmax(x)) for x in lg] == g["tokens"].tolist()
