"""Full-size parity of the BASELINE model configurations on the GPU.

config[2] Llama-3.2-3B, config[3] Llama-3.1-8B and config[4] Qwen3-8B at full
dimensions and depth: per-layer residuals (after_layer0 / after_layer1), the
last-token logits of a 16-token seeded prompt and 8 greedy decode steps
against the C restatement of the reference path (oracle.q8_ref.RefModel,
pinned to the numpy oracle by tests/test_oracle.py, which is pinned to the
reference's own Python).  Long contexts: 2-layer truncations of config[2] at
2048 and of config[4] at 8192 prompt tokens against the numpy oracle
(chunked), then decode steps at those positions.

Weights are made on the GPU (torch RNG, N(0, 0.02) in bf16; norm vectors
1 + N(0, 0.1) so that every norm weight matters) and quantized by the GPU
packer, whose codes are bit-exact with quantize.py (tests/test_gpu_kernels.py);
the checkers read the same packed rows back.  Gates: 2e-2 max-abs and 1e-3
relative L2 on activations and logits, identical greedy tokens.
"""
import numpy as np
import pytest
import torch

from lama32_mojo_b200 import PRESETS, ops
from lama32_mojo_b200.model import Q8Model
from oracle import q8_oracle as O
from oracle import q8_ref as R

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-2


def close(got, ref, what):
    r = O.rel_l2(got, ref)
    m = float(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64)).max())
    assert r <= REL_L2 and m <= MAX_ABS, f"{what}: rel_l2={r:.3e} max_abs={m:.3e}"
    return r


def gpu_weights(m: Q8Model, cfg, seed: int = 0):
    """Loads a seeded synthetic checkpoint made on the GPU into ``m`` and
    returns the host copies the checkers use ({name: packed uint16 rows or
    bf16 bits})."""
    dev = torch.device("cuda", m.device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    host = {}
    for name in cfg.weight_names():
        shp = cfg.tensor_shape(name)
        if len(shp) == 1:
            t = (1.0 + 0.1 * torch.randn(shp, generator=g, device=dev)).to(torch.bfloat16)
            m.load_tensor(name, t, packed=False)
            host[name] = t.view(torch.int16).cpu().numpy().view(np.uint16)
        else:
            w = (torch.randn(shp, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            p = ops.pack_q8(w)
            del w
            m.load_tensor(name, p, packed=True)
            host[name] = p.cpu().numpy().view(np.uint16)
            del p
    torch.cuda.synchronize()
    return host


@pytest.mark.parametrize("cfgname", ["llama-3.2-3b", "llama-3.1-8b", "qwen3-8b"])
def test_full_size_prefill_and_greedy_decode(cuda, cfgname):
    cfg, ocfg = PRESETS[cfgname], O.PRESETS[cfgname]
    m = Q8Model(cfg, device=0, maxlen=64, max_seqs=1, max_tokens=64)
    host = gpu_weights(m, cfg)
    ids = O.random_ids(ocfg, 16, seed=1)
    h0, h1 = m.forward_hidden(ids, 0), m.forward_hidden(ids, 1)
    lg = m.forward(ids)
    toks = [int(np.argmax(lg))]
    am, lg1 = m.decode([toks[-1]], [0], logits=True)  # one-launch decode step, logits out
    toks.append(int(am[0]))
    toks += m.generate([toks[-1]], [0], 7)[:, 0].tolist()
    m.close()

    rm = R.RefModel(ocfg, host, O.inv_freq(ocfg), maxlen=64)
    del host
    rlg, rh = rm.prefill(ids, keep=(0, 1))
    close(h0, rh[0], "after_layer0")
    close(h1, rh[1], "after_layer1")
    close(lg, rlg, "prefill logits")
    want = [int(np.argmax(rlg))]
    rlg1 = rm.token(want[-1])
    close(lg1[0], rlg1, "decode logits")
    want.append(int(np.argmax(rlg1)))
    for _ in range(7):
        want.append(int(np.argmax(rm.token(want[-1]))))
    assert toks == want, (toks, want)


@pytest.mark.parametrize("cfgname,ctx", [("llama-3.2-3b", 2048), ("qwen3-8b", 8192)])
def test_long_context_two_layers(cuda, cfgname, ctx):
    """2-layer truncation at a long prompt: the chunked prefill (tensor-core
    GEMMs and attention), the residuals and logits of the last 16 prompt
    tokens, then 4 greedy decode steps at positions past the prompt."""
    cfg, ocfg = PRESETS[cfgname].replace(layers=2), O.PRESETS[cfgname].replace(layers=2)
    m = Q8Model(cfg, device=0, maxlen=ctx + 16, max_seqs=1, max_tokens=2048)
    host = gpu_weights(m, cfg, seed=3)
    ids = O.random_ids(ocfg, ctx, seed=2)
    m.forward(ids[:-16])
    h1 = m.forward_hidden(ids[-16:], 1)
    lg = m.forward(ids[-16:])
    toks = [int(np.argmax(lg))] + m.generate([int(np.argmax(lg))], [0], 4)[:, 0].tolist()
    m.close()

    orc = O.OracleModel(ocfg, host)
    for i in range(0, ctx - 16, 1024):
        orc.forward_hidden(ids[i:min(i + 1024, ctx - 16)])
    rlg = orc.forward(ids[-16:])
    close(h1, orc.trace["after_layer1"], "after_layer1 (last 16 prompt tokens)")
    close(lg, rlg, "prefill logits")
    want = [int(np.argmax(rlg))]
    for _ in range(4):
        want.append(orc.forward_argmax([want[-1]]))
    assert toks == want, (toks, want)
