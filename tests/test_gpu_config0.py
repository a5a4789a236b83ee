"""config[0] at full size: Llama-3.2-1B dimensions, seed-0 N(0, 0.02) weights
packed bit-exactly by the GPU packer (sha256 of every tensor equals the
reference pack_q8's), 16-token prompt (seed 1): reference-oracle prefill
activations/logits within 2e-2 max-abs / 1e-3 rel-L2 and the 32 greedy decode
tokens identical to the oracle's."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from lama32_mojo_b200 import PRESETS, ops
from lama32_mojo_b200.model import Q8Model
from oracle import q8_oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def test_config0_llama_1b(cuda, golden_dir):
    path = os.path.join(golden_dir, "config0_llama1b.npz")
    g = np.load(path)
    shas = json.load(open(os.path.join(golden_dir, "manifest.json")))["checkpoints"]["llama-3.2-1b"]
    cfg = PRESETS["llama-3.2-1b"]
    m = Q8Model(cfg, maxlen=64)
    bad = []
    for name, w in O.make_bf16_weights(O.PRESETS["llama-3.2-1b"], 0):
        if w.ndim == 2:
            t = torch.from_numpy(w.astype(np.int16)).to(cuda).view(torch.bfloat16)
            p = ops.pack_q8(t)
            if hashlib.sha256(p.cpu().numpy().tobytes()).hexdigest() != shas[name]:
                bad.append(name)
            m.load_tensor(name, p, packed=True)
            del t, p
        else:
            m.load_tensor(name, w, packed=False)
    assert not bad, f"GPU-packed tensors differ from reference pack_q8: {bad[:4]}"
    ids = g["ids"].tolist()
    for L in (0, 1):
        h = m.forward_hidden(ids, L)
        r = O.rel_l2(h, g[f"after_layer{L}"])
        assert r < 1e-3 and np.abs(h - g[f"after_layer{L}"]).max() < 2e-2, (L, r)
    lg = m.forward(ids)
    r = O.rel_l2(lg, g["last_logits"])
    mab = float(np.abs(lg - g["last_logits"]).max())
    assert r < 1e-3 and mab < 2e-2, (r, mab)
    toks = [int(np.argmax(lg))]
    for _ in range(32):
        toks.append(m.forward_argmax([toks[-1]]))
    want = g["tokens"].tolist()
    assert toks == want, (toks, want, g["margins"].tolist())
    m.close()
