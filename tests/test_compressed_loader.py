"""compressed-tensors pack-quantized checkpoints read straight into W4A16 buffers (`from_pack_quantized`,
`install_w4a16_compressed`): host logic only, no kernel runs here. Pinned against the reference's own
`pack_int` and `dequantize_linear` outputs (`tests/golden/golden.pt`, made by `tests/golden/make_golden.py`)."""

import pytest
import torch
from torch import nn

from oracle import w4a16 as ow4


def test_packed_words_pass_through_and_dequantize_like_the_reference(golden):
    from bpt_b200.kernels.w4a16 import from_pack_quantized

    g = golden["pack_int"]
    parts = {"weight_packed": g["packed"], "weight_scale": g["sym_scale"], "weight_shape": torch.tensor([5, 64])}
    qweight, scales, qzeros, group = from_pack_quantized(parts)
    assert qzeros is None and group == 32
    assert torch.equal(qweight, g["packed"])  # compressed-tensors' q + 8 nibbles are this layout's codes
    assert scales.dtype == torch.float16 and torch.equal(scales.to(torch.bfloat16), g["sym_scale"])
    dense = ow4.dequantize_w4a16(ow4.unpack_nibbles_int32(qweight, 64), scales.float(), None, group)
    assert torch.equal(dense.to(torch.bfloat16), g["dense"])  # reference compressed.dequantize_linear


def test_loader_refuses_what_it_cannot_represent():
    from bpt_b200.kernels.w4a16 import from_pack_quantized

    packed = torch.zeros(4, 16, dtype=torch.int32)
    shape = torch.tensor([4, 128])
    ok = torch.full((4, 1), 0.01).to(torch.bfloat16)
    assert from_pack_quantized({"weight_packed": packed, "weight_scale": ok, "weight_shape": shape})[3] == 128
    tiny = torch.full((4, 1), 1e-7).to(torch.bfloat16)  # below fp16's normal range: would change
    with pytest.raises(ValueError, match="fp16"):
        from_pack_quantized({"weight_packed": packed, "weight_scale": tiny, "weight_shape": shape})
    with pytest.raises(NotImplementedError):
        from_pack_quantized({"weight_packed": packed, "weight_scale": ok, "weight_shape": shape,
                             "weight_zero_point": torch.zeros(4, 1)})
    with pytest.raises(ValueError, match="weight_scale"):
        from_pack_quantized({"weight_packed": packed, "weight_scale": torch.ones(4, 3).to(torch.bfloat16),
                             "weight_shape": shape})


class _Attn(nn.Module):
    def __init__(self, h):
        super().__init__()
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            setattr(self, name, nn.Linear(h, h, bias=False))


class _MLP(nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.gate_proj, self.up_proj, self.down_proj = (nn.Linear(h, i, bias=False), nn.Linear(h, i, bias=False),
                                                        nn.Linear(i, h, bias=False))


class _Layer(nn.Module):
    def __init__(self, h, i):
        super().__init__()
        self.self_attn, self.mlp = _Attn(h), _MLP(h, i)


class _Model(nn.Module):
    def __init__(self, layers, h, i):
        super().__init__()
        self.model = nn.Module()
        self.model.layers = nn.ModuleList([_Layer(h, i) for _ in range(layers)])


def _checkpoint(model, group=128, seed=0):
    """A pack-quantized state dict for every decoder linear: random q in [-8, 7] packed as q + 8, bf16 scales."""
    g = torch.Generator().manual_seed(seed)
    state = {}
    for name, mod in model.named_modules():
        if isinstance(mod, nn.Linear):
            out, cols = mod.weight.shape
            q = torch.randint(-8, 8, (out, cols), generator=g)
            state[f"{name}.weight_packed"] = ow4.pack_nibbles_int32((q + 8).to(torch.uint8))
            state[f"{name}.weight_scale"] = (torch.rand(out, cols // group, generator=g) * 0.01 + 1e-3).to(torch.bfloat16)
            state[f"{name}.weight_shape"] = torch.tensor([out, cols])
    return state


CONFIG = {"format": "pack-quantized", "config_groups": {"group_0": {"weights": {"num_bits": 4}}}}


@pytest.mark.parametrize("fuse", [True, False])
def test_install_from_a_compressed_checkpoint(fuse):
    from bpt_b200.kernels.w4a16 import W4A16GateUpMLP, W4A16Linear, install_w4a16_compressed, interleave_rows

    model = _Model(2, 256, 512)
    state = _checkpoint(model)
    install_w4a16_compressed(model, state, CONFIG, fuse_gate_up=fuse)
    for i, layer in enumerate(model.model.layers):
        q = layer.self_attn.q_proj
        assert isinstance(q, W4A16Linear) and q.qzeros is None and q.group == 128
        assert torch.equal(q.qweight, state[f"model.layers.{i}.self_attn.q_proj.weight_packed"])
        if fuse:
            assert isinstance(layer.mlp, W4A16GateUpMLP)
            want = interleave_rows(state[f"model.layers.{i}.mlp.gate_proj.weight_packed"],
                                   state[f"model.layers.{i}.mlp.up_proj.weight_packed"])
            assert torch.equal(layer.mlp.qweight, want) and layer.mlp.qweight.shape == (1024, 32)
            assert torch.equal(layer.mlp.down_proj.qweight, state[f"model.layers.{i}.mlp.down_proj.weight_packed"])
        else:
            assert isinstance(layer.mlp.gate_proj, W4A16Linear) and layer.mlp.down_proj.in_features == 512
    with pytest.raises(ValueError, match="pack-quantized"):
        install_w4a16_compressed(_Model(1, 256, 512), state, {"format": "int-quantized", "config_groups": {}})
