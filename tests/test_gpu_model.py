"""Model-level parity of the B200 path against the golden fixtures made by the
reference's own Python (gen_oracle.py prefill, bench_python.py cached decode)
and against the oracle; plus the reference API semantics (forward /
forward_argmax / n_cached / KV cache full) and the batched and on-device
decode paths.  Gate: per-layer activations and logits within 2e-2 max-abs and
1e-3 relative-L2, identical greedy tokens."""
import json
import os
import struct

import numpy as np
import pytest

from lama32_mojo_b200 import PRESETS
from lama32_mojo_b200._lib import KVCacheFull, Q8Error
from lama32_mojo_b200.model import Q8Model, load_q8
from oracle import q8_oracle as O

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-2


def close(got, ref, rel=REL_L2, mabs=MAX_ABS):
    r = O.rel_l2(got, ref)
    m = float(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64)).max())
    assert r <= rel and m <= mabs, f"rel_l2={r:.3e} max_abs={m:.3e}"
    return r, m


def build(cfgname, packed=False, **kw):
    """Model loaded with the seeded synthetic checkpoint (bf16 -> GPU packer, or
    the oracle-packed rows when packed=True)."""
    cfg = PRESETS[cfgname]
    m = Q8Model(cfg, **kw)
    ocfg = O.PRESETS[cfgname]
    for name, w in O.make_bf16_weights(ocfg, 0):
        if w.ndim == 2 and packed:
            m.load_tensor(name, O.pack_q8(w), packed=True)
        else:
            m.load_tensor(name, w, packed=False)
    return m


@pytest.mark.parametrize("fixture,cfgname", [("tiny_llama_prefill.npz", "tiny-llama"),
                                             ("tiny_llama_untied_prefill.npz", "tiny-llama-untied"),
                                             ("tiny_qwen3_prefill.npz", "tiny-qwen3")])
@pytest.mark.parametrize("packed", [False, True])
def test_prefill_vs_reference_gen_oracle(cuda, golden_dir, fixture, cfgname, packed):
    g = np.load(os.path.join(golden_dir, fixture))
    m = build(cfgname, packed=packed, maxlen=64)
    ids = g["ids"].tolist()
    for L in (0, 1):
        r, _ = close(m.forward_hidden(ids, L), g[f"after_layer{L}"])
        assert r < 1e-5
    assert m.n_cached == 0
    lg = m.forward(ids)
    r, _ = close(lg, g["last_logits"])
    assert r < 1e-5
    assert int(np.argmax(lg)) == int(np.argmax(g["last_logits"]))
    assert m.n_cached == len(ids)
    m.close()


def test_cached_decode_vs_reference_bench_python(cuda, golden_dir):
    g = np.load(os.path.join(golden_dir, "tiny_qwen3_decode.npz"))
    m = build("tiny-qwen3", maxlen=32)
    lg = [m.forward(g["ids"].tolist())]
    toks = [int(np.argmax(lg[0]))]
    for t in g["tokens"][:-1]:
        lg.append(m.forward([int(t)]))
        toks.append(int(np.argmax(lg[-1])))
    close(np.stack(lg), g["logits"])
    assert toks == g["tokens"].tolist()


def test_forward_argmax_and_n_cached_semantics(cuda):
    m = build("tiny-llama-untied", maxlen=12)
    ids = O.random_ids(O.PRESETS["tiny-llama-untied"], 5, seed=3)
    a = m.forward_argmax(ids)
    assert m.n_cached == 5
    m.n_cached = 0  # chat /reset (src/chat.mojo:133-136)
    lg = m.forward(ids)
    assert int(np.argmax(lg)) == a
    m.n_cached = 3  # shrink: re-decode from position 3
    lg2 = m.forward(ids[3:])
    close(lg2, lg, rel=1e-6, mabs=1e-5)
    with pytest.raises(Q8Error):
        m.n_cached = 9  # cannot grow
    with pytest.raises(KVCacheFull):
        m.forward(list(range(8)))  # 5 + 8 > 12
    assert m.n_cached == 5
    m.forward(list(range(7)))  # exactly fills the cache
    assert m.n_cached == 12
    with pytest.raises(KVCacheFull):
        m.forward_argmax([1])
    with pytest.raises(Q8Error):
        m.forward([O.PRESETS["tiny-llama-untied"].vocab])  # token id out of range


@pytest.mark.parametrize("cfgname", ["tiny-llama", "tiny-qwen3"])
def test_incremental_and_chunked_match_oracle(cuda, cfgname):
    ocfg = O.PRESETS[cfgname]
    ck = O.make_q8_checkpoint(ocfg)
    orc = O.OracleModel(ocfg, ck)
    ids = O.random_ids(ocfg, 70, seed=4)
    ref = orc.forward(ids)
    toks, margins, ref_steps = [int(np.argmax(ref))], [], []
    for _ in range(5):
        ref_steps.append(orc.forward([toks[-1]]))
        toks.append(int(np.argmax(ref_steps[-1])))
    # chunked prefill (max_tokens 16 -> 5 chunks), then greedy decode
    m = build(cfgname, maxlen=128, max_tokens=16)
    close(m.forward(ids), ref)
    got = [int(np.argmax(ref))]
    for i in range(5):
        lg = m.forward([got[-1]])
        close(lg, ref_steps[i])
        got.append(int(np.argmax(lg)))
    assert got == toks


@pytest.mark.parametrize("tc_min", [None, "2"])
def test_batched_decode_and_generate(cuda, tc_min, monkeypatch):
    """B=4 host-driven and on-device decode against the oracle; with
    Q8_TC_DECODE_MIN=2 the batch runs the tensor-core layer pipeline (f16
    hi/lo activation rows, decode attention writing them, tcgen05 GEMMs)."""
    if tc_min:
        monkeypatch.setenv("Q8_TC_DECODE_MIN", tc_min)
    cfgname = "tiny-llama-untied"
    ocfg = O.PRESETS[cfgname]
    m = build(cfgname, maxlen=64, max_seqs=4)
    prompts = [O.random_ids(ocfg, n, seed=10 + n) for n in (3, 9, 1, 17)]
    firsts = [m.forward_argmax(p, seq=s) for s, p in enumerate(prompts)]
    # reference: each sequence alone in the oracle
    ck = O.make_q8_checkpoint(ocfg)
    want = []
    for p in prompts:
        o = O.OracleModel(ocfg, ck)
        t = o.forward_argmax(p)
        seqt = []
        for _ in range(4):
            t = o.forward_argmax([t])
            seqt.append(t)
        want.append(seqt)
    assert firsts == [O.OracleModel(ocfg, ck).forward_argmax(p) for p in prompts]
    # two batched host-driven steps (B=4, sequences in a permuted order)
    order = [2, 0, 3, 1]
    cur = {s: firsts[s] for s in range(4)}
    got = {s: [] for s in range(4)}
    for _ in range(2):
        am, lg = m.decode([cur[s] for s in order], order, logits=True)
        for b, s in enumerate(order):
            got[s].append(int(am[b]))
            cur[s] = int(am[b])
            assert int(np.argmax(lg[b])) == int(am[b])
    # two more steps on the device
    toks = m.generate([cur[s] for s in order], order, 2)
    for b, s in enumerate(order):
        got[s] += toks[:, b].tolist()
    for s in range(4):
        assert got[s] == want[s], (s, got[s], want[s])
        assert m.get_n_cached(s) == len(prompts[s]) + 4


def test_decode_rejects_duplicates_and_full(cuda):
    m = build("tiny-qwen3", maxlen=3, max_seqs=2)
    with pytest.raises(Q8Error):
        m.decode([1, 2], [0, 0])
    m.forward([1, 2, 3], seq=1)
    with pytest.raises(KVCacheFull):
        m.decode([1], [1])
    with pytest.raises(KVCacheFull):
        m.generate([1], [0], 4)


def test_missing_weights_is_state_error(cuda):
    m = Q8Model(PRESETS["tiny-qwen3"], maxlen=8)
    with pytest.raises(Q8Error) as e:
        m.forward([1])
    assert "missing tensor" in str(e.value)


def _write_safetensors(path, tensors):
    hdr, blobs, off = {}, [], 0
    for k, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        hdr[k] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


@pytest.mark.parametrize("packed", [True, False])
def test_load_safetensors_packed_and_bf16(cuda, tmp_path, golden_dir, packed):
    """quantize.py output (F16-typed packed rows) and plain bf16 checkpoints both load."""
    cfgname = "tiny-llama"
    ocfg = O.PRESETS[cfgname]
    tensors = {}
    for name, w in O.make_bf16_weights(ocfg, 0):
        if w.ndim == 2 and packed:
            tensors[name] = ("F16", O.pack_q8(w))
        else:
            tensors[name] = ("BF16", w)
    _write_safetensors(tmp_path / "model.safetensors", tensors)
    (tmp_path / "config.json").write_text(json.dumps({
        "hidden_size": ocfg.hidden, "num_hidden_layers": ocfg.layers, "num_attention_heads": ocfg.n_heads,
        "num_key_value_heads": ocfg.n_kv, "head_dim": ocfg.head_dim, "intermediate_size": ocfg.inter,
        "vocab_size": ocfg.vocab, "rms_norm_eps": ocfg.eps, "rope_theta": ocfg.theta,
        "tie_word_embeddings": True, "model_type": "llama",
        "rope_scaling": {"factor": ocfg.rope_factor, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                         "original_max_position_embeddings": 8192, "rope_type": "llama3"}}))
    m = load_q8(str(tmp_path), maxlen=32)
    g = np.load(os.path.join(golden_dir, "tiny_llama_prefill.npz"))
    close(m.forward(g["ids"].tolist()), g["last_logits"])
    # a truncated file is refused with a format error, not a crash
    raw = (tmp_path / "model.safetensors").read_bytes()
    (tmp_path / "model.safetensors").write_bytes(raw[:-64])
    with pytest.raises(Q8Error):
        load_q8(str(tmp_path), maxlen=32)


@pytest.mark.parametrize("cfgname", ["tiny-llama", "tiny-qwen3"])
def test_large_prefill_chunk_and_wide_batch(cuda, cfgname):
    """A 100-token prefill in one chunk (standalone RMSNorm + multi-tile GEMM
    path) and a 12-sequence decode batch (two token tiles) against the oracle."""
    ocfg = O.PRESETS[cfgname]
    ck = O.make_q8_checkpoint(ocfg)
    ids = O.random_ids(ocfg, 100, seed=8)
    m = build(cfgname, maxlen=128, max_tokens=128, max_seqs=12)
    close(m.forward(ids, seq=0), O.OracleModel(ocfg, ck).forward(ids))
    prompts = [O.random_ids(ocfg, 2 + s, seed=30 + s) for s in range(12)]
    for s in range(1, 12):
        m.forward(prompts[s], seq=s)
    toks = [int(t) for t in np.random.default_rng(0).integers(0, ocfg.vocab, 12)]
    am, lg = m.decode(toks, list(range(12)), logits=True)
    for s in range(12):
        o = O.OracleModel(ocfg, ck)
        o.forward(ids if s == 0 else prompts[s])
        close(lg[s], o.forward([toks[s]]))
        assert int(am[s]) == int(np.argmax(lg[s]))


def test_tc_prefill_vs_oracle(cuda):
    """Prefill chunks of >= 128 tokens run the tensor-core GEMMs (tiny-llama-untied
    has every K a multiple of 512): 300 tokens as chunks of 128, 128 and 44
    (tensor core, tensor core, GEMV), then greedy decode; per-layer hidden
    states of a 200-token chunk; all within the f32 oracle gate."""
    cfgname = "tiny-llama-untied"
    ocfg = O.PRESETS[cfgname]
    ck = O.make_q8_checkpoint(ocfg)
    orc = O.OracleModel(ocfg, ck)
    ids = O.random_ids(ocfg, 300, seed=12)
    ref = orc.forward(ids)
    toks = [int(np.argmax(ref))]
    for _ in range(4):
        toks.append(orc.forward_argmax([toks[-1]]))
    m = build(cfgname, maxlen=320, max_tokens=128)
    close(m.forward(ids), ref)
    got = [int(np.argmax(ref))]
    for _ in range(4):
        got.append(m.forward_argmax([got[-1]]))
    assert got == toks
    m.close()
    m2 = build(cfgname, maxlen=256, max_tokens=256)
    o2 = O.OracleModel(ocfg, ck)
    o2.forward(ids[:200])
    for L in (0, 2):
        close(m2.forward_hidden(ids[:200], L), o2.trace[f"after_layer{L}"])
    m2.close()


@pytest.mark.parametrize("cfgname", ["tiny-llama", "tiny-qwen3"])
def test_prefill_attention_context_splits(cuda, cfgname):
    """Prompt chunks of 64 after a growing prefix: the third and fourth chunks
    attend to more than 128 positions, so the tensor-core prefill attention
    splits the context (partials + combine) for head_dim 64 (tiny-llama) and
    128 (tiny-qwen3); logits and greedy tokens against the oracle."""
    ocfg = O.PRESETS[cfgname]
    ck = O.make_q8_checkpoint(ocfg)
    orc = O.OracleModel(ocfg, ck)
    ids = O.random_ids(ocfg, 230, seed=21)
    ref = orc.forward(ids)
    toks = [int(np.argmax(ref))]
    for _ in range(3):
        toks.append(orc.forward_argmax([toks[-1]]))
    m = build(cfgname, maxlen=256, max_tokens=64)
    close(m.forward(ids), ref)
    got = [int(np.argmax(ref))]
    for _ in range(3):
        got.append(m.forward_argmax([got[-1]]))
    assert got == toks
    m.close()


@pytest.mark.parametrize("cfgname", ["small-llama", "small-qwen3", "tiny-llama-untied", "small-pad"])
def test_ring_decode_step_matches_per_op(cuda, cfgname, monkeypatch):
    """The one-launch weight-ring decode step (default for one-sequence greedy
    decode) against the per-operation kernels (Q8_RING=0) on the same
    checkpoint: cached decode logits match the oracle and each other, and
    on-device generation, per-step decode and batched decode give the same
    tokens.  The context grows past several 16-position blocks so that the
    KV append of the ring step is exercised, and the capacity (1024) gives
    the attention 8 context splits per kv head, most of them empty, so that
    the split merge is exercised."""
    ocfg = O.PRESETS[cfgname]
    ck = O.make_q8_checkpoint(ocfg)
    ids = O.random_ids(ocfg, 45, seed=21)
    out = {}
    for ring in ("0", "1"):
        monkeypatch.setenv("Q8_RING", ring)
        m = build(cfgname, maxlen=1024, max_seqs=2)
        m.set_profiling(True)
        m.forward(ids[:-1])
        lg = m.forward([ids[-1]])
        assert ("decode_step" in m.profile()) == (ring == "1"), m.profile().keys()
        m.set_profiling(False)
        t = int(np.argmax(lg))
        gen = m.generate([t], [0], 6)[:, 0].tolist()
        steps = [int(m.decode([gen[-1]], [0])[0])]
        for _ in range(3):
            steps.append(int(m.decode([steps[-1]], [0])[0]))
        m.forward(ids[:5], seq=1)
        am, lgb = m.decode([3, 5], [0, 1], logits=True)
        out[ring] = (lg, gen, steps, lgb)
        m.close()
    o = O.OracleModel(ocfg, ck)
    o.forward(ids[:-1])
    ref = o.forward([ids[-1]])
    close(out["1"][0], ref)
    want = [int(np.argmax(ref))]
    for _ in range(10):
        want.append(o.forward_argmax([want[-1]]))
    assert out["1"][1] == want[1:7]
    assert out["1"][2] == want[7:11]
    r = O.rel_l2(out["1"][0], out["0"][0])
    assert r < 1e-5, r
    assert out["1"][1] == out["0"][1] and out["1"][2] == out["0"][2]
    assert O.rel_l2(out["1"][3], out["0"][3]) < 1e-5


def test_batched_decode_matches_single_sequence_wide(cuda):
    """Hidden 4096 (Llama-3.1-8B width, one layer): decode batches of 3 and 6
    sequences (split-f16 GEMVs with the RMSNorm in front) must give the logits
    of per-sequence decode (the digit GEMV, one token per launch) to f32
    accuracy, and the same greedy tokens."""
    import torch

    from lama32_mojo_b200.config import Config
    cfg = Config("wide-1l", 4096, 1, 32, 8, 128, 1024, 512, 1e-5, 500000.0, "llama3", 8.0, 1.0, 4.0, 8192.0,
                 False, False)
    m = Q8Model(cfg, maxlen=32, max_seqs=6, max_tokens=64)
    try:
        g = torch.Generator(device=cuda).manual_seed(21)
        for name in cfg.weight_names():
            shape = cfg.tensor_shape(name)
            if len(shape) == 2:
                w = (torch.randn(shape, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
            else:
                w = torch.ones(shape, device=cuda, dtype=torch.bfloat16)
            m.load_tensor(name, w, packed=False)
        torch.cuda.synchronize()
        rng = np.random.default_rng(22)
        seqs = list(range(6))
        for s in seqs:
            m.forward(rng.integers(0, cfg.vocab, 3 + s).tolist(), seq=s)
        n0 = [m.get_n_cached(s) for s in seqs]
        ids = rng.integers(0, cfg.vocab, 6).tolist()
        for B in (6, 3):
            am, lg = m.decode(ids[:B], seqs[:B], logits=True)
            for b in range(B):
                m.set_n_cached(n0[b], b)
                am1, lg1 = m.decode([ids[b]], [b], logits=True)
                assert O.rel_l2(lg[b], lg1[0]) < 1e-5, (B, b)
                assert int(am[b]) == int(am1[0])
            for b in range(B):
                m.set_n_cached(n0[b], b)
    finally:
        m.close()


@pytest.mark.parametrize("unit", [1, 0])
def test_device_wait_timeout_fails_the_call(cuda, unit):
    """A bounded device wait that gave up leaves its code in its file's error
    word (unit 1: decode attention, unit 0: tensor-core GEMM).  The model
    calls read both words with their results: the call fails with
    Q8_ERR_TIMEOUT, the word is cleared, and the next call succeeds with the
    oracle's token.  The word is set from the host, so no wait is made to time
    out on the GPU."""
    from lama32_mojo_b200._lib import Q8_ERR_TIMEOUT, lib
    cfgname = "tiny-llama"
    ocfg = O.PRESETS[cfgname]
    orc = O.OracleModel(ocfg, O.make_q8_checkpoint(ocfg))
    ids = O.random_ids(ocfg, 9, seed=21)
    t0 = orc.forward_argmax(ids)
    t1 = orc.forward_argmax([t0])
    m = build(cfgname, maxlen=32)
    assert m.forward_argmax(ids) == t0
    assert lib().q8_debug_set_device_status(unit, Q8_ERR_TIMEOUT) == 0
    with pytest.raises(Q8Error) as e:
        m.decode([t0], [0])
    assert e.value.status == Q8_ERR_TIMEOUT
    assert m.n_cached == len(ids)  # the failed step did not advance the cache
    assert int(m.decode([t0], [0])[0]) == t1
    assert m.n_cached == len(ids) + 1
    assert lib().q8_device_status() == 0
    m.close()
