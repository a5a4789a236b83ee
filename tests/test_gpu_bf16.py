"""bf16-weight path: the reference's non-Q8 run_layer / mm_op
(src/llama_common.mojo:636-780, shells src/llama_gpu.mojo:103-155 and
qwen3_mojo/src/qwen_gpu.mojo) on the GPU.

The product kernel against a float64 product of the same operands; model
prefill and cached decode against the golden fixtures made by the
reference's own gen_oracle.py / bench_python.py on bf16 weights; chunked
prefill, batched decode and config[0] (Llama-3.2-1B) dimensions against the
oracle; the load-time dtype check.  Gates as the Q8 path: 2e-2 max-abs and
1e-3 relative L2 on activations and logits (1e-5 relative L2 against the
fixtures), identical greedy tokens."""
import os

import numpy as np
import pytest
import torch

from lama32_mojo_b200 import PRESETS, ops
from lama32_mojo_b200._lib import Q8Error
from lama32_mojo_b200.model import Q8Model
from oracle import q8_oracle as O

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-2


def close(got, ref, rel=REL_L2, mabs=MAX_ABS):
    r = O.rel_l2(got, ref)
    m = float(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64)).max())
    assert r <= rel and m <= mabs, f"rel_l2={r:.3e} max_abs={m:.3e}"
    return r


def build_bf16(cfgname, seed=0, norm_std=0.1, **kw):
    cfg = PRESETS[cfgname].replace(weights="bf16")
    ocfg = O.PRESETS[cfgname].replace(weights="bf16")
    ck = O.make_bf16_checkpoint(ocfg, seed=seed, norm_std=norm_std)
    m = Q8Model(cfg, **kw)
    for name, w in ck.items():
        m.load_tensor(name, w, packed=False)
    return m, ocfg, ck


@pytest.mark.parametrize("M,K,N,pad", [(1, 512, 1000, 0), (2, 2048, 3072, 0), (3, 1024, 17, 64), (8, 4096, 4096, 0),
                                       (9, 8192, 520, 8), (64, 2048, 512, 0), (130, 1536, 1200, 0)])
def test_mm_bf16_vs_float64(cuda, M, K, N, pad):
    """f32 accumulation over K: error within 1e-5 of sum |x| |w| per output."""
    g = torch.Generator(device=cuda).manual_seed(M * 131 + K + N)
    xb = torch.randn((M, K + pad), generator=g, device=cuda)
    x = xb[:, :K]  # row stride K + pad
    w = (torch.randn((N, K), generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    y = ops.mm_bf16(x, w)
    xd, wd = x.double(), w.double()
    ref = xd @ wd.T
    bound = 1e-5 * (xd.abs() @ wd.abs().T)
    assert bool(((y.double() - ref).abs() <= bound).all())


def test_bf16_prefill_vs_reference_gen_oracle(cuda, golden_dir):
    g = np.load(os.path.join(golden_dir, "tiny_llama_bf16_prefill.npz"))
    m, _, _ = build_bf16("tiny-llama", seed=5, maxlen=64)
    ids = g["ids"].tolist()
    for L in (0, 1):
        assert close(m.forward_hidden(ids, L), g[f"after_layer{L}"]) < 1e-5
    lg = m.forward(ids)
    assert close(lg, g["last_logits"]) < 1e-5
    assert int(np.argmax(lg)) == int(np.argmax(g["last_logits"]))
    m.close()


def test_bf16_cached_decode_vs_reference_bench_python(cuda, golden_dir):
    """Prefill, then the cached decode steps through q8_decode (captured step)."""
    g = np.load(os.path.join(golden_dir, "tiny_qwen3_bf16_decode.npz"))
    m, _, _ = build_bf16("tiny-qwen3", seed=6, maxlen=32)
    lg = [m.forward(g["ids"].tolist())]
    toks = [int(np.argmax(lg[0]))]
    for t in g["tokens"][:-1]:
        am, l1 = m.decode([int(t)], [0], logits=True)
        lg.append(l1[0])
        toks.append(int(am[0]))
    close(np.stack(lg), g["logits"])
    assert toks == g["tokens"].tolist()
    m.close()


@pytest.mark.parametrize("cfgname", ["tiny-llama-untied", "tiny-qwen3"])
def test_bf16_chunked_prefill_and_batched_decode(cuda, cfgname):
    """A 40-token prompt in 16-token chunks, then two sequences decoded as one
    batch (two token rows per product) and with on-device greedy feedback."""
    m, ocfg, ck = build_bf16(cfgname, seed=2, maxlen=128, max_seqs=2, max_tokens=16)
    ids = O.random_ids(ocfg, 40, seed=9)
    orc = O.OracleModel(ocfg, ck)
    close(m.forward(ids), orc.forward(ids))
    m.forward(ids[:5], seq=1)
    o2 = O.OracleModel(ocfg, ck)
    o2.forward(ids[:5])
    first = [orc.forward_argmax([7]), o2.forward_argmax([11])]
    am = m.decode([7, 11], [0, 1])
    assert list(am) == first
    gen = m.generate(first, [0, 1], 5)
    for b, o in enumerate([orc, o2]):
        t, want = first[b], []
        for _ in range(5):
            t = o.forward_argmax([t])
            want.append(t)
        assert gen[:, b].tolist() == want, b
    m.close()


def test_bf16_config0_dims_vs_oracle(cuda):
    """Llama-3.2-1B dimensions (config[0]) with bf16 weights made on the GPU."""
    cfgname = "llama-3.2-1b"
    cfg = PRESETS[cfgname].replace(weights="bf16")
    ocfg = O.PRESETS[cfgname].replace(weights="bf16")
    m = Q8Model(cfg, maxlen=64, max_tokens=64)
    g = torch.Generator(device=cuda).manual_seed(11)
    host = {}
    for name in cfg.weight_names():
        shp = cfg.tensor_shape(name)
        if len(shp) == 1:
            t = (1.0 + 0.1 * torch.randn(shp, generator=g, device=cuda)).to(torch.bfloat16)
        else:
            t = (torch.randn(shp, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
        m.load_tensor(name, t, packed=False)
        host[name] = t.view(torch.int16).cpu().numpy().view(np.uint16)
        del t
    ids = O.random_ids(ocfg, 16, seed=1)
    h1 = m.forward_hidden(ids, 1)
    lg = m.forward(ids)
    toks = [int(np.argmax(lg))] + m.generate([int(np.argmax(lg))], [0], 8)[:, 0].tolist()
    m.close()
    orc = O.OracleModel(ocfg, host)
    rlg = orc.forward(ids)
    close(h1, orc.trace["after_layer1"])
    close(lg, rlg)
    want = [int(np.argmax(rlg))]
    for _ in range(8):
        want.append(orc.forward_argmax([want[-1]]))
    assert toks == want


def test_bf16_model_rejects_packed_rows(cuda):
    cfg = PRESETS["tiny-llama"].replace(weights="bf16")
    m = Q8Model(cfg, maxlen=16)
    w = O.bf16_round(np.random.default_rng(0).standard_normal((cfg.q_dim, cfg.hidden), dtype=np.float32) * 0.02)
    with pytest.raises(Q8Error):
        m.load_tensor("model.layers.0.self_attn.q_proj.weight", O.pack_q8(w), packed=True)
    m.load_tensor("model.layers.0.self_attn.q_proj.weight", w, packed=False)
    m.close()
