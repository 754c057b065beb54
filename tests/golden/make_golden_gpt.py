"""Generate tests/golden/gpt_small.npz by running the REFERENCE's IndexedGPT.

Run once, where a read-only checkout of the reference is available (it is
not present where the tests run), naming it with AIWN_REFERENCE::

    AIWN_REFERENCE=<reference checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_gpt.py

Builds the reference's ``IndexedGPT`` (transformer_validation.py:295-385) at a
small size with dropout 0 on CPU (its IndexedLinear layers take ``_eager``),
runs one forward with targets and ``loss.backward()``, and stores the
state_dict, the token batch, the logits, the loss and every parameter's
gradient.  Tokens are seeded random ids, not text.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch



def _reference_dir() -> str:
    ref = os.environ.get("AIWN_REFERENCE")
    if not ref or not os.path.isdir(os.path.join(ref, "aiwn")):
        raise SystemExit("set AIWN_REFERENCE to the reference checkout (the directory holding aiwn/)")
    return ref


HERE = os.path.dirname(os.path.abspath(__file__))

CFG = dict(vocab_size=65, block_size=32, n_layer=2, n_head=4, n_embd=64, K=16, dropout=0.0)
BATCH = 4


def main():
    sys.path.insert(0, _reference_dir())
    import transformer_validation as tv  # noqa: E402
    torch.manual_seed(123)
    model = tv.IndexedGPT(**CFG)
    g = torch.Generator().manual_seed(7)
    x = torch.randint(0, CFG["vocab_size"], (BATCH, CFG["block_size"]), generator=g)
    y = torch.randint(0, CFG["vocab_size"], (BATCH, CFG["block_size"]), generator=g)
    logits, loss = model(x, y)
    loss.backward()
    out = {f"param:{k}": v.detach().numpy().astype(np.float32) for k, v in model.state_dict().items()}
    out.update({f"grad:{k}": p.grad.detach().numpy().astype(np.float32) for k, p in model.named_parameters()})
    out.update(x=x.numpy(), y=y.numpy(), logits=logits.detach().numpy(), loss=np.float32(loss.item()),
               cfg=np.array([CFG[k] for k in ("vocab_size", "block_size", "n_layer", "n_head", "n_embd", "K")]))
    np.savez_compressed(os.path.join(HERE, "gpt_small.npz"), **out)
    print("wrote gpt_small.npz; loss", loss.item())


if __name__ == "__main__":
    main()
