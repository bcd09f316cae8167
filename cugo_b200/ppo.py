"""PPO update path on the native GEMMs: the actor/critic training step of the
reference's PpoUpdater (python/cugo_ppo50.py:514-745) with residual-MLP networks
whose forward runs on the fused tcgen05 GEMM.

FusedResidualMlp has the parameter layout of the reference's ResidualMlp with
norm="none" (python/cugo_ppo_nets50.py:26-64: inp, blocks.i.fc1/fc2, out), so
PpoActor / OracleCritic state dicts load one to one.  Its autograd function:

  forward   h = inp(x); per block z = fc1(h), u = act(z), h = h + fc2(u);
            out = head(act(h)) -- every Linear is one launch of the fused GEMM
            (bias and residual in the epilogue, fp32 bias, bf16 activations);
  backward  data gradients on the same GEMM with the transposed weights (the
            residual add of dh fused into the epilogue), weight gradients
            dW = dY^T X on cuBLAS (a plain library GEMM: the reduction runs over
            the minibatch), act' and bias sums in torch.

Numerics follow the reference under bf16 autocast: bf16 operands and saved
activations, fp32 accumulation, bf16-rounded weight gradients accumulated into
fp32 parameters.  Data parallelism: gradients of every rank are averaged with one
all-reduce of a flat bucket (NCCL on the GPU box, any torch.distributed backend).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

from .ext import load_extension

FEATURES, ACTIONS, ORACLE_FEATURES = 720, 179, 50
_ACT = {"relu": 1, "silu": 2}


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def _act(z: torch.Tensor, kind: str) -> torch.Tensor:
    return F.silu(z) if kind == "silu" else F.relu(z)


def _act_backward(grad: torch.Tensor, z: torch.Tensor, kind: str) -> torch.Tensor:
    """grad * act'(z), one fused elementwise kernel (bf16 in and out)."""
    if kind == "relu":
        return torch.ops.aten.threshold_backward(grad, z, 0)
    return torch.ops.aten.silu_backward(grad, z)


def _pad4(n: int) -> int:
    return (n + 3) // 4 * 4


def _rows16(t: torch.Tensor) -> torch.Tensor:
    """t as bf16 rows whose stride is a multiple of 8 elements (16 bytes, the TMA
    rule): t itself when it already is, else a zero-padded copy viewed at t's width."""
    if t.dtype == torch.bfloat16 and t.stride(1) == 1 and t.stride(0) % 8 == 0:
        return t
    m, k = t.shape
    z = torch.zeros((m, _pad8(k)), dtype=torch.bfloat16, device=t.device)
    z[:, :k] = t
    return z[:, :k]


class _LinearFn(torch.autograd.Function):
    """One nn.Linear on the tcgen05 kernels, for networks run layer by layer under
    autograd (LayerNorm trunks, the belief head): forward y = x W^T + b (bf16, or fp32
    for a head); backward dX = dY W on the GEMM with the transposed weight, dW = dY^T X
    on the split-K weight-gradient kernel, db = the column sums of dY (fixed order)."""

    @staticmethod
    def forward(ctx, x, weight, bias, ext, out_fp32):
        m, k = x.shape
        n = weight.shape[0]
        xb = _rows16(x)
        wb = _rows16(weight.detach())
        if out_fp32:
            y = torch.empty((m, _pad4(n)), dtype=torch.float32, device=x.device)[:, :n]
            ext.linear(xb, wb, bias.detach(), out=y)
        else:
            y = torch.empty((m, _pad8(n)), dtype=torch.bfloat16, device=x.device)[:, :n]
            ext.linear(xb, wb, bias.detach(), out=y)
        ctx.save_for_backward(xb, wb)
        ctx.ext = ext
        return y

    @staticmethod
    def backward(ctx, dy):
        xb, wb = ctx.saved_tensors
        ext = ctx.ext
        m, k = xb.shape
        n = wb.shape[0]
        dyb = torch.zeros((m, _pad8(n)), dtype=torch.bfloat16, device=dy.device)
        dyb[:, :n] = dy
        dx = None
        if ctx.needs_input_grad[0]:
            wt = torch.zeros((k, _pad8(n)), dtype=torch.bfloat16, device=dy.device)
            wt[:, :n] = wb.t()
            dx = torch.empty((m, _pad8(k)), dtype=torch.bfloat16, device=dy.device)[:, :k]
            ext.linear(dyb[:, :n], wt[:, :n], out=dx)
        dw = torch.empty((n, k), dtype=torch.float32, device=dy.device)
        ext.wgrad_bf16(dyb, xb, dw, n_out=n, n_in=k)
        sums = torch.empty(_pad8(n), dtype=torch.float32, device=dy.device)
        ext.colsum_bf16(dyb, sums)
        return dx, dw, sums[:n], None, None


def _lin(layer: nn.Linear, x: torch.Tensor, ext, out_fp32: bool = False) -> torch.Tensor:
    return _LinearFn.apply(x, layer.weight, layer.bias, ext, out_fp32)


def _layer_norm_bf16(norm: nn.Module, h: torch.Tensor) -> torch.Tensor:
    """nn.LayerNorm as the reference runs it under bf16 autocast: fp32 statistics
    and affine, the result rounded to bf16 for the next Linear."""
    if isinstance(norm, nn.Identity):
        return h
    return F.layer_norm(h.float(), norm.normalized_shape, norm.weight, norm.bias,
                        norm.eps).to(torch.bfloat16)


class _Block(nn.Module):
    def __init__(self, hidden: int, norm: str = "none") -> None:
        super().__init__()
        self.norm = nn.LayerNorm(hidden) if norm == "layer" else nn.Identity()
        self.fc1 = nn.Linear(hidden, hidden)
        self.fc2 = nn.Linear(hidden, hidden)


class _FusedMlpFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, net: "FusedResidualMlp", *params):
        ext = net.ext
        kind, act = net.activation, _ACT[net.activation]
        m = x.shape[0]
        dev = x.device
        ws = [p.detach().to(torch.bfloat16) for p in params[0::2]]
        bs = [p.detach() for p in params[1::2]]  # fp32 biases, used by the epilogue as is
        # Row strides must be multiples of 16 bytes (the TMA rule): the input is read in
        # place when its rows already are (e.g. the 776-wide critic rows that
        # observe_critic_bf16 writes), else copied into padded rows; the input
        # layer's weight is padded likewise.  K stays the true input width.
        k_in = ws[0].shape[1]
        if x.dtype == torch.bfloat16 and x.stride(1) == 1 and x.stride(0) % 8 == 0:
            xb = x[:, :k_in]
        else:
            xp = torch.zeros((m, _pad8(k_in)), dtype=torch.bfloat16, device=dev)
            xp[:, :k_in] = x[:, :k_in]
            xb = xp[:, :k_in]
        w_pad = torch.zeros((ws[0].shape[0], _pad8(k_in)), dtype=torch.bfloat16, device=dev)
        w_pad[:, :k_in] = ws[0]
        h = ext.linear(xb, w_pad[:, :k_in], bs[0])
        saved = [xb]
        for i in range(net.n_blocks):
            w1, b1, w2, b2 = ws[1 + 2 * i], bs[1 + 2 * i], ws[2 + 2 * i], bs[2 + 2 * i]
            z = ext.linear(h, w1, b1)
            u = _act(z, kind)
            h_next = ext.linear(u, w2, b2, residual=h)
            saved += [h, z, u]
            h = h_next
        g = _act(h, kind)
        out_w, out_b = ws[-1], bs[-1]
        n_out = out_w.shape[0]
        ld = (n_out + 3) // 4 * 4
        out = torch.empty((m, ld), dtype=torch.float32, device=dev)
        ext.linear(g, out_w, out_b, out=out[:, :n_out])
        saved += [h, g]
        ctx.save_for_backward(*saved)
        ctx.net = net
        ctx.weights = ws
        return out[:, :n_out].contiguous()

    @staticmethod
    def backward(ctx, dout):
        net = ctx.net
        ext = net.ext
        kind = net.activation
        ws = ctx.weights
        saved = list(ctx.saved_tensors)
        xb = saved[0]
        h_last, g = saved[-2], saved[-1]
        grads_w: list[torch.Tensor] = [None] * len(ws)
        grads_b: list[torch.Tensor] = [None] * len(ws)
        # Head: out = g W^T + b.
        dy = dout.to(torch.bfloat16)
        grads_w[-1] = torch.matmul(dy.t(), g).float()
        grads_b[-1] = dout.sum(0, dtype=torch.float32)
        dg = torch.matmul(dy, ws[-1])  # [M, H]; K = outputs is small: cuBLAS
        dh = _act_backward(dg, h_last, kind)
        for i in reversed(range(net.n_blocks)):
            h, z, u = saved[1 + 3 * i], saved[2 + 3 * i], saved[3 + 3 * i]
            w1, w2 = ws[1 + 2 * i], ws[2 + 2 * i]
            # h_next = h + u W2^T + b2
            grads_w[2 + 2 * i] = torch.matmul(dh.t(), u).float()
            grads_b[2 + 2 * i] = dh.sum(0, dtype=torch.float32)
            du = ext.linear(dh, w2.t().contiguous())              # dh W2, on the tcgen05 GEMM
            dz = _act_backward(du, z, kind)
            grads_w[1 + 2 * i] = torch.matmul(dz.t(), h).float()
            grads_b[1 + 2 * i] = dz.sum(0, dtype=torch.float32)
            dh = ext.linear(dz, w1.t().contiguous(), residual=dh)  # dh + dz W1
        grads_w[0] = torch.matmul(dh.t(), xb).float()
        grads_b[0] = dh.sum(0, dtype=torch.float32)
        out = []
        for gw, gb in zip(grads_w, grads_b):
            out += [gw, gb]
        return (None, None, *out)


class FusedResidualMlp(nn.Module):
    """ResidualMlp whose forward and gradients run on the tcgen05 kernels.
    squeeze: return [M] for a single output (OracleCritic).

    norm "none" (the reference trainer's default): the whole network is one autograd
    function (or one fused kernel for inference).  norm "layer"
    (python/cugo_ppo_nets50.py:20-37: nn.LayerNorm before each block's fc1 and before
    the head): layer by layer under autograd, every Linear on the tcgen05 kernels
    (`_LinearFn`), the LayerNorms and activations in torch; inference keeps an fp32
    residual stream updated in place by the fc2 GEMMs and normalises it with the
    native row LayerNorm."""

    def __init__(self, inputs: int, outputs: int, hidden: int = 512, blocks: int = 3,
                 activation: str = "silu", squeeze: bool = False, zero_out: bool = False,
                 value_bins: int = 0, value_top: float = 640.0, norm: str = "none") -> None:
        super().__init__()
        if activation not in _ACT:
            raise ValueError("activation must be relu or silu")
        if norm not in ("none", "layer"):
            raise ValueError("norm must be none or layer")
        self.activation, self.n_blocks, self.squeeze = activation, blocks, squeeze
        self.norm_kind = norm
        self.inp = nn.Linear(inputs, hidden)
        self.blocks = nn.Sequential(*(_Block(hidden, norm) for _ in range(blocks)))
        self.norm = nn.LayerNorm(hidden) if norm == "layer" else nn.Identity()
        self.out = nn.Linear(hidden, outputs)
        # The reference's norm="none" initialisation: zero residual branches; the
        # actor also zeroes its output layer (python/cugo_ppo_nets50.py:26-31,61-62).
        for b in self.blocks if norm == "none" else ():
            nn.init.zeros_(b.fc2.weight)
            nn.init.zeros_(b.fc2.bias)
        if zero_out:
            nn.init.zeros_(self.out.weight)
            nn.init.zeros_(self.out.bias)
        # OracleCritic's value head (python/cugo_ppo_nets50.py:67-91): one output, or a
        # distribution over symlog-spaced returns whose mean is the value.
        self.stock, self.value_bins = False, value_bins
        if value_bins:
            u = torch.linspace(-1.0, 1.0, value_bins, dtype=torch.float64) * torch.log1p(
                torch.tensor(value_top, dtype=torch.float64))
            self.register_buffer("support", (torch.sign(u) * torch.expm1(u.abs())).float(),
                                 persistent=False)
        self._ext = None

    def value(self, out: torch.Tensor) -> torch.Tensor:
        if not self.value_bins:
            return out.float()
        return (torch.softmax(out.float(), -1) * self.support).sum(-1)

    @property
    def ext(self):
        if self._ext is None:
            self._ext = load_extension()
        return self._ext

    def linears(self) -> list[nn.Linear]:
        return [self.inp] + [l for b in self.blocks for l in (b.fc1, b.fc2)] + [self.out]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        params = [t for l in self.linears() for t in (l.weight, l.bias)]
        x = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        grad = torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in params))
        if self.norm_kind == "layer":
            out = self._forward_layers(x)[0] if grad else self._infer_layer(x, params)
        elif grad:
            out = _FusedMlpFunction.apply(x, self, *params)
        else:
            out = self._infer(x, params)
        return out.squeeze(-1) if self.squeeze and out.shape[-1] == 1 else out

    def forward_hidden(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(output, the trunk's final hidden state before the head's norm), as the
        reference's ResidualMlp.forward_hidden (for the belief head); layer by layer."""
        x = x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
        return self._forward_layers(x)

    def _forward_layers(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Layer by layer under autograd: the reference's module structure under bf16
        autocast (bf16 residual stream, fp32 LayerNorm rounded to bf16)."""
        ext = self.ext
        act = F.silu if self.activation == "silu" else F.relu
        h = _lin(self.inp, _rows16(x[:, :self.inp.in_features]), ext)
        for b in self.blocks:
            u = act(_lin(b.fc1, _layer_norm_bf16(b.norm, h), ext))
            h = h + _lin(b.fc2, u, ext)
        out = _lin(self.out, act(_layer_norm_bf16(self.norm, h)), ext, out_fp32=True)
        return out, h

    def _infer_layer(self, x: torch.Tensor, params: list[torch.Tensor]) -> torch.Tensor:
        """Inference with LayerNorms: an fp32 residual stream updated in place by the
        fc2 GEMMs' epilogues, normalised into bf16 by the native row LayerNorm."""
        ext = self.ext
        act = _ACT[self.activation]
        ws, bs = self._weights(params)
        m, k_pad = x.shape[0], ws[0].shape[1]
        if x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.shape[1] >= k_pad:
            xb = x[:, :k_pad]
        else:
            xb = torch.zeros((m, k_pad), dtype=torch.bfloat16, device=x.device)
            xb[:, :self.inp.in_features] = x[:, :self.inp.in_features]
        hidden = ws[0].shape[0]
        h = torch.empty((m, hidden), dtype=torch.float32, device=x.device)
        ext.linear(xb, ws[0], bs[0], out=h)
        for i, b in enumerate(self.blocks):
            n = ext.layernorm(h, b.norm.weight.detach(), b.norm.bias.detach(), b.norm.eps)
            u = ext.linear(n, ws[1 + 2 * i], bs[1 + 2 * i], act=act)
            ext.linear(u, ws[2 + 2 * i], bs[2 + 2 * i], residual=h, out=h)
        g = ext.layernorm(h, self.norm.weight.detach(), self.norm.bias.detach(), self.norm.eps)
        g = F.silu(g) if self.activation == "silu" else F.relu(g)
        n_out = ws[-1].shape[0]
        out = torch.empty((m, _pad4(n_out)), dtype=torch.float32, device=x.device)
        ext.linear(g, ws[-1], bs[-1], out=out[:, :n_out])
        return out[:, :n_out]

    def _weights(self, params: list[torch.Tensor]):
        """bf16 weights (the input layer's zero-padded to 16-byte rows, contiguous)
        and fp32 biases, converted once per parameter update (tracked by the tensors'
        versions)."""
        key = tuple((p.data_ptr(), p._version) for p in params)
        if getattr(self, "_wkey", None) != key:
            ws = [p.detach().to(torch.bfloat16).contiguous() for p in params[0::2]]
            k_in = ws[0].shape[1]
            w_in = torch.zeros((ws[0].shape[0], _pad8(k_in)), dtype=torch.bfloat16, device=ws[0].device)
            w_in[:, :k_in] = ws[0]
            ws[0] = w_in
            self._wcache = (ws, [p.detach().contiguous() for p in params[1::2]])
            self._wkey = key
        return self._wcache

    def _infer(self, x: torch.Tensor, params: list[torch.Tensor]) -> torch.Tensor:
        """Forward without autograd: one GEMM launch per layer with the activations in
        the epilogues and a scalar head as a row reduction, or, where
        fused_mlp_supported selects it, the whole network in one fused-MLP launch.  The input
        is read in place when its rows are 16-byte multiples at least as wide as the
        zero-padded input weight (e.g. the 776-column rows of observe_critic_bf16)."""
        from .policy import fused_mlp_supported
        ext = self.ext
        act = _ACT[self.activation]
        ws, bs = self._weights(params)
        m, k_pad = x.shape[0], ws[0].shape[1]
        k_in = self.inp.in_features
        if x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.shape[1] >= k_pad:
            xb = x[:, :k_pad]
        else:
            xb = torch.zeros((m, k_pad), dtype=torch.bfloat16, device=x.device)
            xb[:, :k_in] = x[:, :k_in]
        n_out = ws[-1].shape[0]
        if fused_mlp_supported(ws[0].shape[0], self.n_blocks, k_pad, n_out):
            return ext.mlp_fused(xb, ws, bs, act)
        h = ext.linear(xb, ws[0], bs[0], act=act if self.n_blocks == 0 else 0)
        for i in range(self.n_blocks):
            u = ext.linear(h, ws[1 + 2 * i], bs[1 + 2 * i], act=act)
            h = ext.linear(u, ws[2 + 2 * i], bs[2 + 2 * i], residual=h,
                           act_after=act if i == self.n_blocks - 1 else 0)
        if n_out == 1 and ws[-1].shape[1] % 8 == 0 and ws[-1].shape[1] <= 2048:
            # Scalar value head: a row reduction instead of a 256-column GEMM tile.
            w_row = ws[-1].reshape(-1).float()  # the bf16-rounded weights, as the GEMM uses
            return ext.rowdot(h, w_row, bs[-1].float()).unsqueeze(1)
        out = torch.empty((m, (n_out + 3) // 4 * 4), dtype=torch.float32, device=x.device)
        ext.linear(h, ws[-1], bs[-1], out=out[:, :n_out])
        return out[:, :n_out]


# ---- the update's forward and backward without autograd ------------------------------
#
# NativePpoStep runs both networks' forward with the activations kept, the fused
# loss kernel (cugo_b200_ppo_loss) and the backward written out layer by layer,
# every gradient landing in the parameter's .grad buffer directly:
#   head (actor)   dW = dy^T g, db = colsum(dy), dg = dy W on the
#                  tcgen05 GEMM (dy bf16 with rows padded to 184 columns)
#   head (critic)  one kernel: dh, its column sums, dW and db of the scalar head
#   act'(h)        fused with the column sums that are the producing layer's bias
#                  gradient (cugo_b200_colsum_bf16)
#   blocks         dW2 = dh^T u, du = dh W2, dz = du act'(z) (+ db1), dW1 = dz^T h,
#                  dh += dz W1 on the GEMM (residual epilogue), db2 of the block
#                  below = colsum(dh)
#   input layer    dW = dh^T x
# Every dW = dY^T X runs on the split-K tcgen05 kernel (cugo_b200_wgrad_bf16).

_ACT_GRAD = {"relu": 1, "silu": 2}


def _train_weights(net: "FusedResidualMlp"):
    """bf16 weights (the input layer's padded to 16-byte rows), fp32 biases and the
    transposed weights of the backward, cached per parameter version."""
    params = [t for l in net.linears() for t in (l.weight, l.bias)]
    key = tuple((p.data_ptr(), p._version) for p in params)
    if getattr(net, "_tkey", None) != key:
        ws, bs = net._weights(params)
        wt = [w.t().contiguous() for w in ws[1:-1]]
        out_w = ws[-1]
        n_out, hidden = out_w.shape
        wt_out = torch.zeros((hidden, _pad8(n_out)), dtype=torch.bfloat16, device=out_w.device)
        wt_out[:, :n_out] = out_w.t()
        net._tcache = (ws, bs, wt, wt_out)
        net._tkey = key
    return net._tcache


@torch.no_grad()
def train_forward(net: "FusedResidualMlp", x: torch.Tensor):
    """The forward of a training step, keeping what the backward reads: returns
    (out fp32 [m, n_out] (rows padded to 16 bytes), saved activations)."""
    ext = net.ext
    kind = net.activation
    ws, bs, _, _ = _train_weights(net)
    m = x.shape[0]
    k_in = net.inp.in_features
    if x.dtype == torch.bfloat16 and x.stride(1) == 1 and x.stride(0) % 8 == 0:
        xb = x[:, :k_in]
    else:
        xp = torch.zeros((m, _pad8(k_in)), dtype=torch.bfloat16, device=x.device)
        xp[:, :k_in] = x[:, :k_in]
        xb = xp[:, :k_in]
    h = ext.linear(xb, ws[0][:, :k_in], bs[0])
    saved = {"x": xb, "h": [], "z": [], "u": []}
    for i in range(net.n_blocks):
        z = torch.empty_like(h)
        u = ext.linear_pre(h, ws[1 + 2 * i], bs[1 + 2 * i], _ACT[kind], z)  # u = act(z), z kept
        saved["h"].append(h)
        saved["z"].append(z)
        saved["u"].append(u)
        h = ext.linear(u, ws[2 + 2 * i], bs[2 + 2 * i], residual=h)
    saved["h_last"] = h
    n_out = ws[-1].shape[0]
    out = torch.empty((m, (n_out + 3) // 4 * 4), dtype=torch.float32, device=x.device)
    if n_out == 1:
        g = None
        ext.rowdot(h if kind == "none" else _act(h, kind), ws[-1].reshape(-1).float(), bs[-1].float(),
                   out=out[:, 0])
    else:
        g = _act(h, kind)
        ext.linear(g, ws[-1], bs[-1], out=out[:, :n_out])
    saved["g"] = g
    return out[:, :n_out], saved


def _grad(p: torch.Tensor) -> torch.Tensor:
    if p.grad is None:
        p.grad = torch.zeros_like(p)
    return p.grad


@torch.no_grad()
def train_backward(net: "FusedResidualMlp", saved: dict, dy: torch.Tensor | None = None,
                   dv: torch.Tensor | None = None) -> None:
    """Writes every parameter's gradient into its .grad: dy bf16 [m, >= n_out] (rows
    of 16-byte multiples; columns past n_out zero) for a matrix head, dv fp32 [m]
    for a one-output head."""
    ext = net.ext
    kind = net.activation
    act = _ACT_GRAD[kind]
    ws, _, wt, wt_out = _train_weights(net)
    lin = net.linears()
    h_last = saved["h_last"]
    m, hidden = h_last.shape
    dh = torch.empty_like(h_last)
    # Gradient of the bias of the layer that produced h_last.
    below = lin[-2]
    if dv is not None:  # one-output head: one pass over h_last
        ext.scalar_head_backward(dv, ws[-1].reshape(-1), h_last, act, dh, _grad(below.bias),
                                 _grad(lin[-1].weight).view(-1), _grad(lin[-1].bias))
    else:
        n_out = lin[-1].out_features
        ext.wgrad_bf16(dy, saved["g"], _grad(lin[-1].weight), n_out=n_out)
        sums = torch.empty(dy.shape[1], dtype=torch.float32, device=dy.device)
        ext.colsum_bf16(dy, sums)
        _grad(lin[-1].bias).copy_(sums[:n_out])
        dg = ext.linear(dy[:, :n_out], wt_out[:, :n_out])
        ext.colsum_bf16(dg, _grad(below.bias), z=h_last, act=act, dz=dh)
    for i in reversed(range(net.n_blocks)):
        h, z, u = saved["h"][i], saved["z"][i], saved["u"][i]
        fc1, fc2 = lin[1 + 2 * i], lin[2 + 2 * i]
        ext.wgrad_bf16(dh, u, _grad(fc2.weight))
        du = ext.linear(dh, wt[2 * i + 1])                      # dh W2
        dz = torch.empty_like(du)
        ext.colsum_bf16(du, _grad(fc1.bias), z=z, act=act, dz=dz)
        ext.wgrad_bf16(dz, h, _grad(fc1.weight))
        dh = ext.linear(dz, wt[2 * i], residual=dh)              # dh + dz W1
        ext.colsum_bf16(dh, _grad(lin[2 * i].bias))              # the layer below's bias
    ext.wgrad_bf16(dh, saved["x"], _grad(lin[0].weight))


def fused_actor(hidden: int = 512, blocks: int = 3, norm: str = "none") -> FusedResidualMlp:
    """PpoActor's shape: 720 features -> 179 logits, zero-initialised output layer."""
    return FusedResidualMlp(FEATURES, ACTIONS, hidden, blocks, "silu", zero_out=True, norm=norm)


class FusedBeliefHead(nn.Module):
    """The reference's BeliefHead (python/cugo_ppo_nets50.py:94-105, the same parameter
    names: net.0 LayerNorm, net.1 and net.3 Linear): logits of which of the 50 cards
    the opponent holds, from the actor trunk's final hidden state; the Linears on
    the tcgen05 kernels (`_LinearFn`), LayerNorm and GELU in torch, as the reference
    runs them under bf16 autocast."""

    def __init__(self, inputs: int, width: int | None = None) -> None:
        super().__init__()
        width = width or inputs
        self.net = nn.Sequential(nn.LayerNorm(inputs), nn.Linear(inputs, width), nn.GELU(),
                                 nn.Linear(width, ORACLE_FEATURES))
        self._ext = None

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        if self._ext is None:
            self._ext = load_extension()
        t = F.gelu(_lin(self.net[1], _layer_norm_bf16(self.net[0], h), self._ext))
        return _lin(self.net[3], t, self._ext, out_fp32=True)


def card_plane(masks: torch.Tensor) -> torch.Tensor:
    """int64 card masks [N] as an fp32 [N, 50] 0/1 plane (the belief targets)."""
    bits = torch.arange(ORACLE_FEATURES, device=masks.device)
    return ((masks.view(-1, 1) >> bits) & 1).float()


def two_hot(y: torch.Tensor, support: torch.Tensor) -> torch.Tensor:
    """[N, bins] target whose mean over `support` (increasing) is y clamped to its
    range: weight split between the two bins around y in proportion to distance
    (the value-distribution target of the reference's OracleCritic with bins)."""
    y = torch.minimum(torch.maximum(y, support[0]), support[-1])
    upper = torch.searchsorted(support, y.contiguous()).clamp(1, support.numel() - 1)
    lower = upper - 1
    lo_v, hi_v = support[lower], support[upper]
    w_upper = ((y - lo_v) / (hi_v - lo_v)).clamp(0.0, 1.0)
    out = torch.zeros((y.numel(), support.numel()), dtype=torch.float32, device=y.device)
    out.scatter_(1, lower.view(-1, 1), (1.0 - w_upper).view(-1, 1))
    out.scatter_add_(1, upper.view(-1, 1), w_upper.view(-1, 1))
    return out


STOCK_FEATURES = 8 * 50  # one-hot planes of the next 8 stock draws


def fused_critic(hidden: int = 512, blocks: int = 3, value_bins: int = 0,
                 value_top: float = 640.0, stock: bool = False, norm: str = "none") -> FusedResidualMlp:
    """OracleCritic's shape (python/cugo_ppo_nets50.py:67-91): 770 inputs, or 1,170
    with the stock planes -> one value (or value_bins logits of the return
    distribution)."""
    inputs = FEATURES + ORACLE_FEATURES + (STOCK_FEATURES if stock else 0)
    net = FusedResidualMlp(inputs, value_bins or 1, hidden, blocks, "silu",
                           squeeze=not value_bins, value_bins=value_bins, value_top=value_top,
                           norm=norm)
    net.stock = stock
    return net


def critic_input(features: torch.Tensor, opp_hand: torch.Tensor,
                 stock: torch.Tensor | None = None) -> torch.Tensor:
    """[features, one-hot plane of the opponent's hand, (one-hot planes of the next
    8 stock draws, stock_indexed's packing, 0xFF = none)] as bf16 (the reference's
    _critic_input, python/cugo_ppo50.py:478-482).  The rows are written into a buffer padded to a multiple of 8 columns (zeros
    past the last input) and returned as a view of the input width, so the first
    GEMM reads them in place (its TMA rows must be 16-byte multiples)."""
    dev = opp_hand.device
    bits = torch.arange(ORACLE_FEATURES, device=dev)
    width = FEATURES + ORACLE_FEATURES + (STOCK_FEATURES if stock is not None else 0)
    out = torch.empty((features.shape[0], _pad8(width)), dtype=torch.bfloat16, device=dev)
    out[:, :FEATURES] = features
    out[:, FEATURES:FEATURES + ORACLE_FEATURES] = (opp_hand.view(-1, 1) >> bits) & 1
    if stock is not None:
        cards = (stock.view(-1, 1) >> torch.arange(0, 64, 8, device=dev)) & 0xFF
        out[:, FEATURES + ORACLE_FEATURES:width] = (cards.unsqueeze(-1) == bits).flatten(1)
    out[:, width:] = 0
    return out[:, :width]


def allreduce_gradients(params: list[torch.Tensor], world: int) -> None:
    """Averages the gradients of `params` over the ranks with one all-reduce of a
    flat bucket (the data-parallel step of the update; a no-op for one rank)."""
    finish_allreduce(start_allreduce(params, world))


def flat_gradients(params: list[torch.Tensor]) -> torch.Tensor:
    """Makes every parameter's .grad a view into one flat fp32 buffer (returned), so a
    data-parallel step all-reduces the gradients in place, with no gather into a
    bucket and no copy back.  The gradients must then be written, not replaced
    (zero_grad with set_to_none=False)."""
    total = sum(p.numel() for p in params)
    flat = torch.zeros(total, dtype=torch.float32, device=params[0].device)
    off = 0
    for p in params:
        p.grad = flat[off:off + p.numel()].view_as(p)
        off += p.numel()
    return flat


class _Bucket:
    """A flat gradient bucket whose all-reduce is in flight; `grads` are the
    tensors to copy the result back into (None when the bucket is their storage)."""

    def __init__(self, grads: list[torch.Tensor] | None, flat: torch.Tensor, work, world: int) -> None:
        self.grads, self.flat, self.work, self.world = grads, flat, work, world


def start_allreduce(params: list[torch.Tensor], world: int,
                    flat: torch.Tensor | None = None) -> "_Bucket | None":
    """Starts the all-reduce of the gradients of `params` without waiting: on NCCL
    the collective runs on the communicator's stream after the work queued so far,
    so the caller's next kernels (the other network's backward) overlap it.  `flat`:
    the buffer of flat_gradients(params), reduced in place; otherwise the gradients
    are gathered into a new bucket.  None for one rank."""
    if world <= 1:
        return None
    if flat is not None:
        return _Bucket(None, flat, dist.all_reduce(flat, async_op=True), world)
    grads = [p.grad for p in params if p.grad is not None]
    bucket = torch.cat([g.reshape(-1) for g in grads])
    return _Bucket(grads, bucket, dist.all_reduce(bucket, async_op=True), world)


def finish_allreduce(bucket: "_Bucket | None") -> None:
    """Waits for a bucket's all-reduce and leaves the averaged gradients in place."""
    if bucket is None:
        return
    bucket.work.wait()
    bucket.flat.div_(bucket.world)
    if bucket.grads is None:
        return
    off = 0
    for g in bucket.grads:
        g.copy_(bucket.flat[off:off + g.numel()].view_as(g))
        off += g.numel()


@dataclass
class Minibatch:
    features: torch.Tensor  # bf16 [B, 720]
    legal: torch.Tensor     # bool [B, 179]
    actions: torch.Tensor   # int64 [B]
    logp_old: torch.Tensor  # fp32 [B]
    opp_hand: torch.Tensor  # int64 [B]
    adv: torch.Tensor       # fp32 [B]
    ret: torch.Tensor       # fp32 [B]
    stock: torch.Tensor | None = None  # int64 [B], for a critic with stock planes

    def tensors(self) -> tuple[torch.Tensor, ...]:
        return tuple(t for t in (self.features, self.legal, self.actions, self.logp_old,
                                 self.opp_hand, self.adv, self.ret, self.stock) if t is not None)


class PpoStep:
    """One PPO minibatch update (python/cugo_ppo50.py:558-623, the plain policy
    target): clipped surrogate, entropy bonus, value loss (smooth L1, or the
    cross-entropy against the two-hot return for a critic with value bins),
    optionally the belief head's binary cross-entropy on the opponent's hand,
    gradient clipping per network, the optimizer step and the running statistics
    (policy, value, entropy, KL, clip fraction, count, belief loss)."""

    def __init__(self, actor: nn.Module, critic: nn.Module, optimizer: torch.optim.Optimizer,
                 clip: float = 0.2, value_coef: float = 0.5, grad_clip: float = 1.0,
                 world: int = 1, belief: nn.Module | None = None, belief_coef: float = 0.0) -> None:
        self.actor, self.critic, self.optimizer = actor, critic, optimizer
        self.clip, self.value_coef, self.grad_clip, self.world = clip, value_coef, grad_clip, world
        self.belief, self.belief_coef = belief, belief_coef
        self.groups = [list(actor.parameters()), list(critic.parameters())]
        if belief is not None:
            self.groups.append(list(belief.parameters()))
        dev = next(actor.parameters()).device
        self.entropy_coef = torch.zeros((), device=dev)
        self.sums = torch.zeros(7, device=dev)
        self.last_kl = torch.zeros((), device=dev)  # the latest minibatch's KL estimate

    def losses(self, mb: Minibatch):
        belief_loss = None
        if self.belief is not None:
            out, hidden = self.actor.forward_hidden(mb.features)
            logits = out.float()
            belief_loss = F.binary_cross_entropy_with_logits(self.belief(hidden).float(),
                                                             card_plane(mb.opp_hand))
        else:
            logits = self.actor(mb.features).float()
        stock = mb.stock if getattr(self.critic, "stock", False) else None
        value = self.critic(critic_input(mb.features, mb.opp_hand, stock)).float()
        log_probs = torch.log_softmax(logits.masked_fill(~mb.legal, -1.0e30), dim=1)
        new_logp = log_probs.gather(1, mb.actions.unsqueeze(1)).squeeze(1)
        log_ratio = new_logp - mb.logp_old
        ratio = log_ratio.exp()
        surrogate = torch.minimum(ratio * mb.adv, ratio.clamp(1 - self.clip, 1 + self.clip) * mb.adv)
        policy_loss = -surrogate.mean()
        entropy = -(log_probs.exp() * log_probs).sum(1).mean()
        if getattr(self.critic, "value_bins", 0):
            target = two_hot(mb.ret, self.critic.support)
            value_loss = -(target * torch.log_softmax(value, -1)).sum(-1).mean()
        else:
            value_loss = F.smooth_l1_loss(value, mb.ret)
        return policy_loss, value_loss, entropy, ratio, log_ratio, belief_loss

    def step(self, mb: Minibatch) -> None:
        """One update, eager (every kernel launched from Python)."""
        self.optimizer.zero_grad(set_to_none=False)
        policy_loss, value_loss, entropy, ratio, log_ratio, belief_loss = self.losses(mb)
        loss = policy_loss - self.entropy_coef * entropy + self.value_coef * value_loss
        if belief_loss is not None:
            loss = loss + self.belief_coef * belief_loss
        loss.backward()
        allreduce_gradients([p for g in self.groups for p in g], self.world)
        for group in self.groups:
            nn.utils.clip_grad_norm_(group, self.grad_clip, foreach=True)
        self.optimizer.step()
        with torch.no_grad():
            kl = ((ratio - 1) - log_ratio).mean()
            self.last_kl.copy_(kl)
            bl = belief_loss.detach() if belief_loss is not None else torch.zeros_like(kl)
            self.sums += torch.stack((policy_loss.detach(), value_loss.detach(), entropy.detach(), kl,
                                      ((ratio - 1).abs() > self.clip).float().mean(),
                                      torch.ones_like(kl), bl))


class NativePpoStep(PpoStep):
    """PpoStep without autograd for two FusedResidualMlp networks (the actor with a
    matrix head, a scalar critic): train_forward of both, the fused loss kernel,
    train_backward of both writing the gradients, then the same clipping, optimizer
    step and statistics.  Gradients of the hidden layers' weights are fp32 products
    of the bf16 operands (autograd's path rounds them to bf16)."""

    def __init__(self, actor: FusedResidualMlp, critic: FusedResidualMlp,
                 optimizer: torch.optim.Optimizer, clip: float = 0.2, value_coef: float = 0.5,
                 grad_clip: float = 1.0, world: int = 1) -> None:
        super().__init__(actor, critic, optimizer, clip, value_coef, grad_clip, world)
        self.stats = torch.zeros(5, device=self.sums.device)
        self.ones = torch.ones(1, device=self.sums.device)
        # Each network's gradients live in one flat buffer, the bucket of its all-reduce.
        self.flat = {"actor": flat_gradients(list(actor.parameters())),
                     "critic": flat_gradients(list(critic.parameters()))} if world > 1 else {}
        # On one GPU the critic's forward and backward run on a second stream beside
        # the actor's: the two networks are independent up to the loss, and the
        # kernels of one fill the SMs the other's tail waves and small launches leave.
        self.side = torch.cuda.Stream(self.sums.device) if world == 1 and self.sums.is_cuda else None

    @staticmethod
    def supports(actor: nn.Module, critic: nn.Module) -> bool:
        return (isinstance(actor, FusedResidualMlp) and isinstance(critic, FusedResidualMlp)
                and actor.norm_kind == "none" and critic.norm_kind == "none"
                and not critic.value_bins and critic.out.out_features == 1
                and actor.out.out_features == ACTIONS and actor.inp.in_features == FEATURES)

    def step(self, mb: Minibatch) -> None:
        ext = self.actor.ext
        stock = mb.stock if getattr(self.critic, "stock", False) else None
        main, side = torch.cuda.current_stream(), self.side
        if side is not None:  # the critic's forward beside the actor's
            side.wait_stream(main)
            with torch.cuda.stream(side):
                value, c_saved = train_forward(self.critic,
                                               critic_input(mb.features, mb.opp_hand, stock))
            logits, a_saved = train_forward(self.actor, mb.features)
            main.wait_stream(side)
            value.record_stream(main)
        else:
            logits, a_saved = train_forward(self.actor, mb.features)
            value, c_saved = train_forward(self.critic, critic_input(mb.features, mb.opp_hand, stock))
        b = logits.shape[0]
        dy = torch.empty((b, _pad8(ACTIONS)), dtype=torch.bfloat16, device=logits.device)
        dv = torch.empty(b, dtype=torch.float32, device=logits.device)
        ext.ppo_loss(logits, mb.legal, mb.actions, mb.logp_old, mb.adv, value, mb.ret, self.clip,
                     self.entropy_coef, self.value_coef, dy, dv, self.stats)
        if side is not None:  # the two backwards side by side
            side.wait_stream(main)
            dv.record_stream(side)
            with torch.cuda.stream(side):
                train_backward(self.critic, c_saved, dv=dv)
            train_backward(self.actor, a_saved, dy=dy)
            main.wait_stream(side)
        else:
            # Data parallel: the critic's gradients are all-reduced while the actor's
            # backward runs (two buckets, the same collective order on every rank).
            train_backward(self.critic, c_saved, dv=dv)
            critic_bucket = start_allreduce(list(self.critic.parameters()), self.world,
                                            self.flat.get("critic"))
            train_backward(self.actor, a_saved, dy=dy)
            actor_bucket = start_allreduce(list(self.actor.parameters()), self.world,
                                           self.flat.get("actor"))
            finish_allreduce(critic_bucket)
            finish_allreduce(actor_bucket)
        for group in self.groups:
            nn.utils.clip_grad_norm_(group, self.grad_clip, foreach=True)
        self.optimizer.step()
        self.last_kl.copy_(self.stats[3])
        self.sums[:5] += self.stats
        self.sums[5:6] += self.ones


def make_ppo_step(actor: nn.Module, critic: nn.Module, optimizer: torch.optim.Optimizer,
                  clip: float = 0.2, value_coef: float = 0.5, grad_clip: float = 1.0,
                  world: int = 1, belief: nn.Module | None = None,
                  belief_coef: float = 0.0) -> PpoStep:
    """The native step where both networks are FusedResidualMlp (norm "none", scalar
    critic, no belief head), else the autograd one."""
    if belief is None and NativePpoStep.supports(actor, critic):
        return NativePpoStep(actor, critic, optimizer, clip, value_coef, grad_clip, world)
    return PpoStep(actor, critic, optimizer, clip, value_coef, grad_clip, world, belief, belief_coef)


class GraphedPpoStep:
    """PpoStep captured once as a CUDA graph over static minibatch buffers and
    replayed per minibatch, as the reference's PpoUpdater._run does
    (python/cugo_ppo50.py:625-657): three warm-up steps on a side stream, the
    weights and optimizer moments restored, one captured step.  The optimizer must
    be capturable (torch.optim.Adam(..., capturable=True)); data-parallel runs
    (world > 1) step eagerly."""

    def __init__(self, step: PpoStep, template: Minibatch) -> None:
        self.step = step
        self.static = Minibatch(*(t.clone() for t in template.tensors()))
        self.graph: torch.cuda.CUDAGraph | None = None

    def _capture(self) -> None:
        st = self.step
        params = [p for g in st.groups for p in g]
        saved_sums = st.sums.clone()
        weights = [p.detach().clone() for p in params]
        moments = {p: {k: v.clone() for k, v in st.optimizer.state[p].items() if torch.is_tensor(v)}
                   for p in params if p in st.optimizer.state}
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                st.step(self.static)
        torch.cuda.current_stream().wait_stream(side)
        with torch.no_grad():  # undo the warm-up updates in place (the graph keeps these tensors)
            for p, w in zip(params, weights):
                p.copy_(w)
            for p in params:
                before = moments.get(p)
                for k, v in st.optimizer.state[p].items():
                    if torch.is_tensor(v):
                        v.copy_(before[k]) if before is not None else v.zero_()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            st.step(self.static)
        st.sums.copy_(saved_sums)

    def __call__(self, mb: Minibatch) -> None:
        if self.step.world > 1:
            self.step.step(mb)
            return
        for dst, src in zip(self.static.tensors(), mb.tensors(), strict=True):
            dst.copy_(src)
        if self.graph is None:
            self._capture()
        self.graph.replay()
