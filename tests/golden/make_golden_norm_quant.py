"""Write tests/golden/norm_quant.pt: outputs of the REFERENCE's `kernels.reference.rms_norm_int8`
(ish-codes-magic/bytes-per-token, `src/fastserve/kernels/reference.py:44-55`) on small seeded inputs, to pin the
CPU oracle `oracle/norm_quant.py`.

Run where the reference is importable (its `src/` directory on the path), e.g.

    python tests/golden/make_golden_norm_quant.py /path/to/bytes-per-token/src

The reference is never needed at test time: the tests read only the committed `norm_quant.pt`.
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch


def main(src: str) -> None:
    sys.path.insert(0, src)
    from fastserve.engine.model import RMSNorm
    from fastserve.kernels import reference

    gold: dict[str, dict] = {}

    def entry(name, x, w, eps, **extra):
        codes, scale = reference.rms_norm_int8(x, w, eps)
        gold[name] = {"x": x, "weight": w, "eps": torch.tensor(eps, dtype=torch.float64), "codes": codes,
                      "scale": scale, **extra}

    # the reference test's known values (tests/kernels/test_reference.py:27-31)
    entry("kat", torch.tensor([[3.0, -4.0, 0.0, 0.0]]), torch.ones(4), 0.0)

    g = torch.Generator().manual_seed(0)
    x = torch.randn(9, 100, generator=g)
    x[4] = 0.0  # an all-zero token: scale 1e-12, codes 0
    entry("f32_zero_row", x, torch.ones(100), 1e-6)

    x = (torch.randn(5, 7, 64, generator=g) * 3).to(torch.bfloat16)
    w = (torch.rand(64, generator=g) + 0.5).to(torch.bfloat16)
    norm = RMSNorm(64, eps=1e-6)
    norm.weight.data = w.float()
    entry("bf16_3d", x, w, 1e-6, model_norm=norm(x.float()))

    x = (torch.randn(3, 2048, generator=g) * 3).to(torch.float16)
    w = (torch.rand(2048, generator=g) + 0.5).to(torch.float16)
    entry("f16_2048", x, w, 1e-6)

    x = torch.randn(4, 1000, generator=g).to(torch.bfloat16)
    w = torch.rand(1000, generator=g) + 0.5  # an f32 weight on bf16 activations
    entry("bf16_x_f32_w", x, w, 1e-5)

    # the decoder layer's residual add in front (engine/model.py:109-111): the bf16 sum is what gets normalized
    h = (torch.randn(6, 2048, generator=g) * 2).to(torch.bfloat16)
    delta = torch.randn(6, 2048, generator=g).to(torch.bfloat16)
    w = (torch.rand(2048, generator=g) + 0.5).to(torch.bfloat16)
    entry("residual", h + delta, w, 1e-6, h=h, delta=delta)

    out_path = Path(__file__).with_name("norm_quant.pt")
    torch.save(gold, out_path)
    print(f"wrote {out_path} ({out_path.stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_norm_quant.py <reference src directory>")
    main(sys.argv[1])
