"""Shared helpers of the parity tests: seeded inputs and the oracle's view of them."""
import numpy as np
import torch

from oracle import oracle as O


def rand_int8(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)


def rand_scales(n, seed, mag):
    g = torch.Generator().manual_seed(seed)
    return torch.rand(n, generator=g) * mag


def bits(t):
    return O.to_bits(t)


def from_bits(b, dtype):
    return O.from_bits(b, dtype)


def assert_bits_equal(got, want_bits, what):
    gb = bits(got.cpu())
    if not np.array_equal(gb, want_bits):
        diff = np.argwhere(gb != want_bits)
        raise AssertionError(f"{what}: {len(diff)} of {gb.size} differ, first at {diff[:4].tolist()}")


def rel_err(got, want):
    got = got.double()
    want = want.double()
    return ((got - want).abs() / (want.abs() + 1e-3)).max().item()


def q_off(got_q, want_q):
    d = np.abs(got_q.astype(np.int32) - want_q.astype(np.int32))
    return int(d.max()) if d.size else 0
