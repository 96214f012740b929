"""Generates tests/golden/dtypes.safetensors and tests/golden/dtypes_expected.npz.

The .safetensors file is written by the `safetensors` package (an implementation
of the format independent of this repository and of the reference), with one
tensor per dtype the reference reads (SafeTensors.kt:23-30, :136-170) and
values chosen for the conversion's edge cases: every binary16 bit pattern,
bfloat16 specials and random patterns, float64 values exactly halfway between
two float32s, integers above 2^24 that round, the limits of each integer type,
and a metadata map.  The .npz holds torch's float32 conversion of each tensor
(``tensor.to(torch.float32)``), an independent statement of the values the
reference's readInto produces.

Run: python tests/golden/make_safetensors_golden.py
"""
from __future__ import annotations

import os

import numpy as np
import torch
from safetensors.torch import save_file

HERE = os.path.dirname(os.path.abspath(__file__))


def tensors() -> dict:
    rng = np.random.default_rng(20240611)
    out = {}
    out["halves"] = torch.from_numpy(np.arange(65536, dtype=np.uint16).view(np.float16).copy()).reshape(256, 256)
    bf = np.concatenate([
        np.array([0x0000, 0x8000, 0x3F80, 0xBF80, 0x7F80, 0xFF80, 0x7F7F, 0x0001, 0x8001, 0x0080, 0x4049],
                 np.uint16),
        rng.integers(0, 65536, 4085, dtype=np.uint16)])
    out["bfloats"] = torch.from_numpy(bf.astype(np.int16)).view(torch.bfloat16)
    f32 = np.concatenate([np.array([0.0, -0.0, 1.5, -2.25, 1e-10, 7.0, np.inf, -np.inf, 3.4028235e38, 1e-45],
                                   np.float32), rng.standard_normal(1014).astype(np.float32)])
    out["floats"] = torch.from_numpy(f32).reshape(32, 32)
    one = 1.0
    ties = [one + 2.0 ** -24, one + 3 * 2.0 ** -24, -(one + 2.0 ** -24), 2.0 ** 128, -2.0 ** 129, 1e-46, 2.0 ** -150,
            3 * 2.0 ** -151, 0.1, 1e300, -1e-300, 0.0, -0.0]
    f64 = np.concatenate([np.array(ties), rng.standard_normal(499) * 1e3, np.nextafter(np.float64(1.0), 2.0, dtype=np.float64)[None]])
    out["doubles"] = torch.from_numpy(f64.astype(np.float64))
    i64 = np.concatenate([np.array([0, -1, 2**24 + 1, 2**24 + 3, -(2**24 + 1), 2**53 + 1, 2**62 + 2**38,
                                    np.iinfo(np.int64).max, np.iinfo(np.int64).min], np.int64),
                          rng.integers(-2**62, 2**62, 247, dtype=np.int64)])
    out["longs"] = torch.from_numpy(i64)
    i32 = np.concatenate([np.array([0, -1, 2**24 + 1, 2**24 + 3, 2**31 - 1, -2**31, 16777217], np.int32),
                          rng.integers(-2**31, 2**31 - 1, 249, dtype=np.int32)])
    out["ints"] = torch.from_numpy(i32)
    out["shorts"] = torch.from_numpy(np.arange(-32768, 32768, 257, dtype=np.int16))
    out["bytes"] = torch.from_numpy(np.arange(-128, 128, dtype=np.int8))
    out["ubytes"] = torch.from_numpy(np.arange(0, 256, dtype=np.uint8))
    out["flags"] = torch.from_numpy(np.array([True, False, True, True, False]))
    out["scalar"] = torch.tensor(2.5, dtype=torch.float32)
    return out


def main() -> None:
    t = tensors()
    save_file(t, os.path.join(HERE, "dtypes.safetensors"), metadata={"format": "pt", "note": "kotensor dtype fixture"})
    expected = {name: x.to(torch.float32).reshape(-1).numpy() for name, x in t.items()}
    np.savez_compressed(os.path.join(HERE, "dtypes_expected.npz"), **expected)


if __name__ == "__main__":
    main()
