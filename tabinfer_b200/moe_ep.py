"""Expert-parallel int3 MoE FFN (tb_moe_ep_*): the LFM2.5 MoE of
models/lfm25.js (router, idxGemv3, MOECOMBINE) with its experts spread over P
ranks, one process per GPU.  The reference keeps every expert on one device
(lfm25.js:824-830); the exchange is this library's own: token rows go straight
into the owning rank's IPC-mapped arena over NVLink and the expert outputs come
back the same way, so one forward is six kernels and no library collective.
The result is bit-identical to moe_ffn_int3 with all experts on one GPU."""
import ctypes

import torch

from ._lib import LIB
from .ops import Context, TabInferError, _p, default_context


class MoeEP:
    """Rank `rank` of P.  Experts [rank*nE/P, (rank+1)*nE/P) live here; T <=
    t_max tokens per rank and call.  For P > 1, exchange handle() across the
    ranks (any host channel) and call connect() with all P in rank order."""

    def __init__(self, P, rank, n_experts, top_k, hidden, inter, t_max, device=0, ctx: Context = None):
        self.P, self.rank, self.nE, self.K, self.H, self.I = P, rank, n_experts, top_k, hidden, inter
        self.device = torch.device("cuda", device)
        self.ctx = ctx or default_context(device)
        h = ctypes.c_void_p()
        self.ctx.check(LIB.tb_moe_ep_create(self.ctx.h, P, rank, n_experts, top_k, hidden, inter, t_max,
                                            ctypes.byref(h)), "moe_ep_create")
        self.h = h
        self._experts = None

    @property
    def local_experts(self):
        n = self.nE // self.P
        return range(self.rank * n, (self.rank + 1) * n)

    def handle(self):
        buf = ctypes.create_string_buffer(64)
        self.ctx.check(LIB.tb_moe_ep_handle(self.h, buf), "moe_ep_handle")
        return buf.raw

    def connect(self, handles):
        blob = b"".join(bytes(x) for x in handles)
        if len(blob) != 64 * self.P:
            raise TabInferError("need %d handles" % self.P)
        self.ctx.check(LIB.tb_moe_ep_connect(self.h, ctypes.c_char_p(blob)), "moe_ep_connect")

    def set_experts(self, w1, w3, w2):
        """This rank's experts as (planes, scales) pairs, layout of moe_ffn_int3
        with nE/P experts; kept referenced."""
        self._experts = (w1, w3, w2)
        self.ctx.check(LIB.tb_moe_ep_set_experts(self.h, _p(w1[0]), _p(w1[1]), _p(w3[0]), _p(w3[1]), _p(w2[0]),
                                                 _p(w2[1])), "moe_ep_set_experts")

    def forward(self, x_out, x_in, idx, wt):
        """x_out += MoE FFN of x_in routed by (idx, wt) from moe_router (global ids)."""
        T = idx.shape[0]
        if idx.shape[1] != self.K or x_in.shape != (T, self.H) or x_out.shape != (T, self.H):
            raise TabInferError("moe_ep forward: shapes")
        self.ctx.check(LIB.tb_moe_ep_forward(self.h, _p(x_out), _p(x_in), _p(idx), _p(wt), T), "moe_ep_forward")
        return x_out

    def close(self):
        if getattr(self, "h", None):
            LIB.tb_moe_ep_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
