"""Helpers shared by the GPU tests (host <-> device bit-pattern moves)."""
import numpy as np
import torch


def to_dev(bits):
    """uint16 numpy bit patterns -> CUDA bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).cuda()


def to_bits(x):
    """bf16 tensor -> uint16 numpy bit patterns."""
    return x.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def same_bits(a, b):
    return torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))
