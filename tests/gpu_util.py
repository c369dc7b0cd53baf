"""Helpers shared by the GPU parity tests."""
import numpy as np
import torch
import torch.nn.functional as F

from oracle import moe_oracle as mo


def to_dev(bits, device="cuda"):
    """uint16 BF16 bits (numpy) -> BF16 CUDA tensor."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def to_bits(t):
    """BF16 tensor -> uint16 bits (numpy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def f32(t):
    return t.detach().float().cpu().numpy()


def torch_route(x, gate, top_k, normalize):
    """The reference's route() body (qwen.py:147-152) run with torch on the device."""
    logits = F.linear(x, gate)
    probs = F.softmax(logits, dim=-1, dtype=torch.float32)
    w, sel = torch.topk(probs, top_k, dim=-1)
    if normalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return logits, sel, w.to(x.dtype)


def torch_expert_forward(x, g, u, d):
    """The reference's expert_forward() (qwen.py:87-90) with torch on the device."""
    return F.linear(F.silu(F.linear(x, g)) * F.linear(x, u), d)


def assert_close_bf16(actual_bits, expected_bits, rtol=2e-2, atol=2e-2):
    a = mo.bf16_to_f32(actual_bits)
    e = mo.bf16_to_f32(expected_bits)
    np.testing.assert_allclose(a, e, rtol=rtol, atol=atol)
