"""CPU stand-ins for the codec kernels, for tests of host logic only.

The block store's INT8/INT4 paths call the CUDA codec (``quantize_tensor``,
``PackedTensor.dequantize``).  Tests that exercise only the store's host
bookkeeping on CPU swap those two for the oracle's numpy restatement, which is
bit-exact with the reference (tests/test_oracle_golden.py), with
:func:`use_oracle_codec`.  FP16 and EVICTED need no kernel and keep the
package's own code.
"""

import torch

from anchorkv_b200 import backend as B
from anchorkv_b200.policy import CacheMode
from oracle import codec as OC

_PACKAGE_QUANTIZE = B.quantize_tensor


def oracle_quantize(tensor, mode, *, group_size=64):
    mode = CacheMode(getattr(mode, "value", mode))
    if mode in (CacheMode.FP16, CacheMode.EVICTED):
        return _PACKAGE_QUANTIZE(tensor, mode, group_size=group_size)
    bits = 8 if mode is CacheMode.INT8 else 4
    payload, scales = OC.quantize_tensor(tensor.detach().float().numpy(), bits, group_size)
    return B.PackedTensor(mode, tuple(tensor.shape), tensor.dtype, torch.from_numpy(payload),
                          torch.from_numpy(scales), group_size, tensor.numel())


def oracle_dequantize(self, *, dtype=None, device=None):
    if self.mode is CacheMode.EVICTED or self.payload is None:
        raise RuntimeError("evicted tensors cannot be materialized")
    out_dtype = self.original_dtype if dtype is None else dtype
    if self.mode is CacheMode.FP16:
        return self.payload.to(out_dtype).reshape(self.shape)
    bits = 8 if self.mode is CacheMode.INT8 else 4
    vals = OC.dequantize_tensor(self.payload.numpy(), self.scales.numpy(), bits, self.group_size,
                                self.original_numel)
    return torch.from_numpy(vals).reshape(self.shape).to(out_dtype)


def use_oracle_codec(monkeypatch):
    monkeypatch.setattr(B, "quantize_tensor", oracle_quantize)
    monkeypatch.setattr(B.PackedTensor, "dequantize", oracle_dequantize)
