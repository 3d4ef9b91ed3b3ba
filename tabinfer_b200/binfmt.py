"""The `.cpu.bin` ternary model container on the device (native/docs/FORMAT.md).

Host-side mirror of the reference reader, native/crates/n2-core/src/binfmt.rs:
`Container.open(path)` (binfmt.rs:104) validates the header exactly as the
reference does and streams the blob into one device allocation;
`ternary(name)` / `f32s(name)` / `embed(name)` (binfmt.rs:298-341) hand back
zero-copy torch tensors in the kernels' layout -- Q2_0_g64 codes u8 [N, K/4]
and f32 scales [N, K/64] for `tb_gemv_tern_q2g64`, f16 bits for the embedding
table, f32 norm weights.  Errors raise TabInferError with the reference's
wording.  Tensors are views of the container's device memory: they are valid
until `close()`.
"""
import ctypes

import torch

from ._lib import LIB, P, BinTensor, BIN_TERN, BIN_EMBED_F16, BIN_F32
from .ops import TabInferError, default_context

KINDS = {BIN_TERN: "tern", BIN_EMBED_F16: "embed_f16", BIN_F32: "f32"}


def check(path):
    """None when the container's header is valid (Container::assemble + validate,
    binfmt.rs:155-257), else the reason.  Needs no GPU."""
    buf = ctypes.create_string_buffer(512)
    rc = LIB.tb_bin_check(str(path).encode(), buf, len(buf))
    return None if rc == 0 else buf.value.decode()


class _DevArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(int(s) for s in shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


class Container:
    def __init__(self, h, device):
        self.h = h
        self.device = device

    @classmethod
    def open(cls, path, device=0):
        ctx = default_context(device)
        h = P()
        ctx.check(LIB.tb_bin_open(ctx.h, str(path).encode(), ctypes.byref(h)), "bin_open %s" % path)
        return cls(h, device)

    def close(self):
        if self.h:
            LIB.tb_bin_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def blob_bytes(self):
        return int(LIB.tb_bin_blob_bytes(self.h))

    def _info(self, name=None, index=None):
        info = BinTensor()
        if name is not None:
            rc = LIB.tb_bin_find(self.h, name.encode(), ctypes.byref(info))
            if rc:
                raise TabInferError("%s: not in container" % name)
        else:
            rc = LIB.tb_bin_info(self.h, int(index), ctypes.byref(info))
            if rc:
                raise TabInferError("tensor index %d out of range" % index)
        return info

    def names(self):
        return [self._info(index=i).name.decode() for i in range(LIB.tb_bin_count(self.h))]

    def info(self, name):
        i = self._info(name)
        return {"kind": KINDS[i.kind], "N": i.N, "K": i.K, "shape": list(i.shape[:i.ndim]),
                "bytes": i.bytes, "scales_bytes": i.scales_bytes, "blob_offset": i.blob_offset}

    def _view(self, ptr, shape, typestr, dtype):
        return torch.as_tensor(_DevArray(ptr, shape, typestr), device="cuda:%d" % self.device).view(dtype)

    def ternary(self, name):
        """(codes u8 [N, K/4], scales f32 [N, K/64]) -- Container::ternary, binfmt.rs:298-312."""
        i = self._info(name)
        if i.kind != BIN_TERN:
            raise TabInferError("%s: expected `tern`, found `%s`" % (name, KINDS[i.kind]))
        codes = self._view(i.data, (i.N, i.K // 4), "|u1", torch.uint8)
        scales = self._view(i.scales, (i.N, i.K // 64), "<f4", torch.float32)
        return codes, scales

    def f32s(self, name):
        """f32 tensor (norm weights) -- Container::f32s, binfmt.rs:314-321."""
        i = self._info(name)
        if i.kind != BIN_F32:
            raise TabInferError("%s: expected `f32`, found `%s`" % (name, KINDS[i.kind]))
        return self._view(i.data, (i.bytes // 4,), "<f4", torch.float32).view(*i.shape[:i.ndim])

    def embed(self, name):
        """f16 bit patterns [rows, dim] as int16 -- the table embed_row decodes (binfmt.rs:323-341)."""
        i = self._info(name)
        if i.kind != BIN_EMBED_F16:
            raise TabInferError("%s: expected `embed_f16`, found `%s`" % (name, KINDS[i.kind]))
        return self._view(i.data, (i.bytes // 2,), "<i2", torch.int16).view(*i.shape[:i.ndim])
