"""Reader of the golden vectors written by tests/golden/make_golden.py."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


class Golden:
    def __init__(self, name):
        self.z = np.load(GOLDEN / f"{name}.npz")

    def has(self, key):
        return key in self.z.files

    def str(self, key):
        return str(self.z[key])

    def int(self, key):
        return int(self.z[key])

    def t(self, key):
        """Tensor stored under `key` (bf16 restored from its raw bits)."""
        if key not in self.z.files:
            return None
        arr = self.z[key]
        dt = str(self.z[key + ".dtype"])
        if dt == "bfloat16":
            return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16)
        return torch.from_numpy(arr.copy())
