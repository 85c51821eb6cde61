"""Write tests/golden/golden.pt: outputs of the REFERENCE itself (ish-codes-magic/bytes-per-token,
`src/fastserve`) on small seeded inputs, to pin the CPU oracle (`oracle/`).

Run where the reference is importable (its `src/` directory on the path), e.g.

    python tests/golden/make_golden.py /path/to/bytes-per-token/src

The reference is never needed at test time: the tests read only the committed `golden.pt`.
Every entry names the reference function that produced it.
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch


def main(src: str) -> None:
    sys.path.insert(0, src)
    from fastserve.engine.config import ModelConfig
    from fastserve.engine.kv_cache import PagedKVCache
    from fastserve.kernels import reference
    from fastserve.kernels.kv_attention import default_split
    from fastserve.kv.quant import store
    from fastserve.kv.sizing import TensorQuant
    from fastserve.quant.compressed import dequantize_linear, pack_int, unpack_int
    from fastserve.quant.formats import E4M3, round_to_format
    from fastserve.quant.rtn import IntSpec, fake_quantize, quantize

    gold: dict[str, torch.Tensor | dict] = {}

    # ---- W4A16 pieces: rtn asymmetric grid (rtn.py:77-114), fake quantize, linear ----------------------------
    g = torch.Generator().manual_seed(0)
    w = torch.randn(16, 256, generator=g) * 0.02
    w[3, :128] = 0.0  # an all-zero group
    w[5, 128:] = w[5, 128:].abs() + 0.01  # an all-positive group: the range is stretched to 0
    spec = IntSpec(4, "group", 128, symmetric=False)
    q, scale, zero = quantize(w, spec)
    x = torch.randn(3, 256, generator=g)
    w_hat = fake_quantize(w, spec)
    gold["rtn_asym"] = {
        "w": w,
        "q": q,
        "scale": scale,
        "zero": zero,
        "w_hat": w_hat,
        "x": x,
        "y": torch.nn.functional.linear(x, w_hat),
    }

    # ---- compressed-tensors int32 packing (compressed.py:25-53) and symmetric dequant (:56-69) -----------------
    qs = torch.randint(-8, 8, (5, 64), generator=g, dtype=torch.int8)
    qs[0, :2] = torch.tensor([-8, 7])
    sym_scale = torch.rand(5, 2, generator=g).to(torch.bfloat16)
    gold["pack_int"] = {
        "q": qs,
        "packed": pack_int(qs, 4),
        "packed37": pack_int(qs[:, :37], 4),
        "unpacked": unpack_int(pack_int(qs, 4), 64, 4),
        "sym_scale": sym_scale,
        "dense": dequantize_linear(
            {"weight_packed": pack_int(qs, 4), "weight_scale": sym_scale, "weight_shape": torch.tensor([5, 64])}
        ),
    }

    # ---- KIVI storage and decode attention (reference.py:103-224) -------------------------------------------
    def random_kv(batch, heads, tokens, dim, seed):
        gg = torch.Generator().manual_seed(seed)
        k = torch.randn(batch, heads, tokens, dim, generator=gg)
        k[..., 3] += 20.0
        return k, torch.randn(batch, heads, tokens, dim, generator=gg)

    for bits in (4, 8, 16):
        k, v = random_kv(2, 2, 64, 16, seed=bits)
        kv = reference.quantize_kv(k, v, bits, group=32)
        qq = torch.randn(2, 4, 16, generator=torch.Generator().manual_seed(7))
        lengths = torch.tensor([64, 33])
        out, lse = reference.decode_attention(qq, kv, lengths, scale=0.25)
        k_hat, v_hat = reference.dequantize_kv(kv)
        entry = {"k": k, "v": v, "q": qq, "lengths": lengths, "out": out, "lse": lse, "k_hat": k_hat, "v_hat": v_hat}
        for name in ("k_codes", "v_codes", "k_scale", "k_zero", "v_scale", "v_zero"):
            if getattr(kv, name) is not None:
                entry[name] = getattr(kv, name)
        entry["merged"] = reference.merge_partials(out, lse)
        gold[f"kivi{bits}"] = entry

    # ---- split/merge with ragged rows and an empty split (reference.py:186-211) ------------------------------
    k, v = random_kv(3, 2, 96, 16, seed=11)
    qq = torch.randn(3, 4, 16, generator=torch.Generator().manual_seed(6))
    lengths = torch.tensor([96, 40, 5])
    outs, lses = [], []
    for start in (0, 32, 64):
        seen = (lengths - start).clamp(0, 32)
        o, s_ = reference.partial_attention(qq, k[:, :, start : start + 32], v[:, :, start : start + 32], seen, 0.25)
        outs.append(o)
        lses.append(s_)
    gold["splits"] = {
        "k": k,
        "v": v,
        "q": qq,
        "lengths": lengths,
        "outs": torch.stack(outs, 2),
        "lses": torch.stack(lses, 2),
        "merged": reference.merge_partials(torch.stack(outs, 2), torch.stack(lses, 2)),
    }

    # ---- FP8 storage (kv/quant.py:44-45) and the from-scratch E4M3 rounding (formats.py:43-52) ---------------
    xf = torch.cat([torch.randn(512, generator=g) * 10.0 ** torch.randint(-4, 3, (512,), generator=g),
                    torch.tensor([1000.0, -1000.0, 448.0, 464.0, 0.0])])
    gold["fp8"] = {
        "x": xf,
        "stored": store(xf.reshape(1, 1, 1, -1), TensorQuant(8, kind="fp8")).reshape(-1),
        "rounded": round_to_format(xf.clamp(-448, 448), E4M3),
    }

    # ---- symmetric INT8 per token (kv/quant.py:35-48 -> rtn.py:82-85) ---------------------------------------
    xi = torch.randn(64, 128, generator=g) * 3
    xi[7] = 0.0
    qi, si, _ = quantize(xi, IntSpec(8, "channel", symmetric=True))
    gold["int8_token"] = {
        "x": xi,
        "q": qi,
        "scale": si,
        "stored": store(xi.reshape(1, 1, 64, 128), TensorQuant(8, axis="token", group=128, symmetric=True)).reshape(64, 128),
    }

    # ---- the paged gather (engine/kv_cache.py:140-169) -------------------------------------------------------
    cfg = ModelConfig(
        vocab_size=16, hidden_size=32, intermediate_size=64, num_layers=1, num_heads=4, num_kv_heads=2,
        head_dim=16, rope_theta=1e6, rms_norm_eps=1e-6, tie_word_embeddings=True,
    )
    cache = PagedKVCache(cfg, num_blocks=8, block_size=4, dtype=torch.float32, device="cpu")
    cache.k[0].copy_(torch.randn(cache.k[0].shape, generator=g))
    cache.reserve("a", 11)
    cache.reserve("b", 6)
    cache.free("b")
    cache.reserve("c", 9)
    meta = cache.prepare(["a", "c"], torch.tensor([[10], [8]]))
    gold["paged_gather"] = {
        "pool": cache.k[0].clone(),
        "block_table": meta.block_table,
        "kv_len": torch.tensor(meta.kv_len),
        "write_blocks": meta.write_blocks,
        "write_offsets": meta.write_offsets,
        "gathered": cache._gather(cache.k[0], meta),
    }

    # ---- paged decode attention through the reference pieces ----------------------------------------------
    # FP8 pool (kv/quant.py:44-45 codes), random block table, ragged lengths; the reference reads it through
    # PagedKVCache._gather and reference.partial_attention. Codes are stored as uint8 bytes.
    nb, bs, hkv, d, b = 24, 4, 2, 16, 3
    kf = torch.randn(nb, bs, hkv, d, generator=g) * 2
    vf = torch.randn(nb, bs, hkv, d, generator=g)
    k_scale, v_scale = 0.5, 0.25
    k_codes = (kf / k_scale).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    v_codes = (vf / v_scale).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
    perm = torch.randperm(nb, generator=g)[: b * 5].reshape(b, 5)
    lengths = torch.tensor([17, 4, 9])
    cache = PagedKVCache(cfg, num_blocks=nb, block_size=bs, dtype=torch.float32, device="cpu")
    cache.k[0].copy_(k_codes.view(torch.float8_e4m3fn).float() * k_scale)
    cache.v[0].copy_(v_codes.view(torch.float8_e4m3fn).float() * v_scale)
    from fastserve.engine.kv_cache import PagedMeta

    meta = PagedMeta(write_blocks=perm[:, :1], write_offsets=perm[:, :1] * 0, block_table=perm, kv_len=17)
    qq = torch.randn(b, 4, d, generator=g)
    out, lse = reference.partial_attention(qq, cache._gather(cache.k[0], meta), cache._gather(cache.v[0], meta),
                                           lengths, 0.25)
    gold["paged_fp8"] = {
        "k_codes": k_codes, "v_codes": v_codes, "k_scale": torch.tensor(k_scale), "v_scale": torch.tensor(v_scale),
        "block_table": perm.to(torch.int32), "lengths": lengths.to(torch.int32), "q": qq, "out": out, "lse": lse,
        "block_size": torch.tensor(bs),
    }

    # ---- default_split (kv_attention.py:178-187) ---------------------------------------------------------------
    cases = [(1, 8, 32768), (64, 8, 8192), (1, 8, 100), (3, 8, 1000), (8, 8, 32768), (32, 8, 4096), (2, 2, 7)]
    gold["default_split"] = {"cases": torch.tensor(cases), "split": torch.tensor([default_split(*c) for c in cases])}

    out_path = Path(__file__).with_name("golden.pt")
    torch.save(gold, out_path)
    print(f"wrote {out_path} ({out_path.stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference src directory>")
    main(sys.argv[1])
