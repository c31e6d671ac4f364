"""a 2-layer MLP's forward and backward (6 products per step) on the library's kernels.

    H  = bf16(relu(X W1))                  cairn_b200_gemm, OUT_BF16 with ReLU fused
    Y  = H W2                              cairn_b200_gemm, f32 out
    loss, dY = mean((Y - T)^2), bf16(2 (Y - T) / n)          cairn_b200_mse_grad
    dW2 = H^T dY                           cairn_b200_gemm, A transposed, f32 out
    dH  = bf16(dY W2^T) where H > 0        cairn_b200_gemm_relu_grad, B transposed, ReLU's backward fused
    dW1 = X^T dH                           cairn_b200_gemm, A transposed, f32 out
    dX  = dH W1^T                          cairn_b200_gemm, B transposed, f32 out

The backward is the one derive grad writes for a dense layer (compiler/derive/gradients.py:1-11; d_x = d_out w^T,
d_w = x^T d_out), on the tensor cores instead of sequential host loops. `MLPLoss` wraps the step as a
torch.autograd.Function so that `loss.backward()` runs these kernels.
"""

from __future__ import annotations

import torch

from ._lib import ACT_RELU, BF16, OUT_BF16, OUT_STORE_F32, CairnError, check, lib

ERR_ARG = 7


class MLPWorkspace:
    """The step's intermediates for one shape, allocated once and reused by every step."""

    def __init__(self, batch: int, d_in: int, d_hidden: int, d_out: int, device: torch.device):
        self.shape = (batch, d_in, d_hidden, d_out)
        bf, f32 = torch.bfloat16, torch.float32
        self.h = torch.empty(batch, d_hidden, dtype=bf, device=device)
        self.y = torch.empty(batch, d_out, dtype=f32, device=device)
        self.dy = torch.empty(batch, d_out, dtype=bf, device=device)
        self.loss = torch.empty(1, dtype=f32, device=device)
        self.dw2 = torch.empty(d_hidden, d_out, dtype=f32, device=device)
        self.dh = torch.empty(batch, d_hidden, dtype=bf, device=device)
        self.dw1 = torch.empty(d_in, d_hidden, dtype=f32, device=device)
        self.dx = torch.empty(batch, d_in, dtype=f32, device=device)


def mlp_step(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, t: torch.Tensor, ws: MLPWorkspace | None = None,
             stream: int | None = None) -> MLPWorkspace:
    """One forward + backward of loss = mean((relu(x w1) w2 - t)^2): x (B x D), w1 (D x H), w2 (H x O) bf16, t (B x O)
    f32. Queued on `stream` (torch's current stream by default); the results are the workspace's tensors."""
    batch, d_in = x.shape
    d_hidden, d_out = w2.shape
    if w1.shape != (d_in, d_hidden) or t.shape != (batch, d_out):
        raise CairnError(1, "mlp_step: shapes disagree")
    if any(v.dtype != torch.bfloat16 for v in (x, w1, w2)) or t.dtype != torch.float32:
        raise CairnError(ERR_ARG, "mlp_step: x, w1, w2 bf16 and t f32")
    if ws is None:
        ws = MLPWorkspace(batch, d_in, d_hidden, d_out, x.device)
    L = lib()
    s = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    B, D, Hd, O = batch, d_in, d_hidden, d_out
    p = lambda v: v.data_ptr()  # noqa: E731
    check(L.cairn_b200_gemm(s, BF16, B, Hd, D, p(x), 0, p(w1), 0, p(ws.h), OUT_BF16, None, ACT_RELU), "mlp fwd 1")
    check(L.cairn_b200_gemm(s, BF16, B, O, Hd, p(ws.h), 0, p(w2), 0, p(ws.y), OUT_STORE_F32, None, 0), "mlp fwd 2")
    check(L.cairn_b200_mse_grad(s, B * O, p(ws.y), p(t), p(ws.dy), p(ws.loss)), "mlp loss")
    check(L.cairn_b200_gemm(s, BF16, Hd, O, B, p(ws.h), 1, p(ws.dy), 0, p(ws.dw2), OUT_STORE_F32, None, 0), "mlp dW2")
    check(L.cairn_b200_gemm_relu_grad(s, BF16, B, Hd, O, p(ws.dy), 0, p(w2), 1, p(ws.dh), p(ws.h)), "mlp dH")
    check(L.cairn_b200_gemm(s, BF16, D, Hd, B, p(x), 1, p(ws.dh), 0, p(ws.dw1), OUT_STORE_F32, None, 0), "mlp dW1")
    check(L.cairn_b200_gemm(s, BF16, B, D, Hd, p(ws.dh), 0, p(w1), 1, p(ws.dx), OUT_STORE_F32, None, 0), "mlp dX")
    return ws


class HostFeed:
    """Batches from pinned host memory for a run of steps. Each batch (x, t) is copied on the feed's own stream into
    one of `depth` device buffer sets while the step before computes from another, so a training loop's input copies
    overlap its products instead of preceding them; a set is refilled only after the step that read it has run."""

    def __init__(self, batch: int, d_in: int, d_out: int, device: torch.device, depth: int = 2):
        self.sets = [[torch.empty(batch, d_in, dtype=torch.bfloat16, device=device),
                      torch.empty(batch, d_out, dtype=torch.float32, device=device), None] for _ in range(depth)]
        self.copy = torch.cuda.Stream(device)
        self.calls = 0

    def put(self, x_host: torch.Tensor, t_host: torch.Tensor):
        """Queues the batch's copies; returns (x, t, ready, slot): the device tensors, the event that marks them
        copied, and the slot to hand back to `done`."""
        slot = self.calls % len(self.sets)
        self.calls += 1
        x, t, free = self.sets[slot]
        if x_host.shape != x.shape or t_host.shape != t.shape or x_host.dtype != x.dtype or t_host.dtype != t.dtype:
            raise CairnError(ERR_ARG, "HostFeed.put: x and t of the feed's shapes (x bf16, t f32)")
        if free is not None:
            self.copy.wait_event(free)
        with torch.cuda.stream(self.copy):
            x.copy_(x_host, non_blocking=True)
            t.copy_(t_host, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(self.copy)
        return x, t, ready, slot

    def done(self, slot: int, stream: torch.cuda.Stream) -> None:
        """The step that reads `slot` is queued on `stream`: the set may be refilled once it has run."""
        e = torch.cuda.Event()
        e.record(stream)
        self.sets[slot][2] = e


def step_from_host(feed: HostFeed, x_host: torch.Tensor, t_host: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                   ws: MLPWorkspace, loss_host: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
    """One step whose batch and target come from host memory and whose loss goes back to it, all queued on `stream`
    (torch's current stream by default) behind the feed's copies; returns at once."""
    stream = torch.cuda.current_stream(w1.device) if stream is None else stream
    x, t, ready, slot = feed.put(x_host, t_host)
    stream.wait_event(ready)
    mlp_step(x, w1, w2, t, ws, stream.cuda_stream)
    with torch.cuda.stream(stream):
        loss_host.copy_(ws.loss, non_blocking=True)
    feed.done(slot, stream)


def mlp_flops(batch: int, d_in: int, d_hidden: int, d_out: int) -> float:
    """Six products of 2 * batch * d_in * d_hidden (= 2 * batch * d_hidden * d_out when d_in = d_out) flops each."""
    return 2.0 * batch * d_hidden * (3 * d_in + 3 * d_out)


class MLPLoss(torch.autograd.Function):
    """loss = mean((relu(x w1) w2 - t)^2) with the forward and the backward on the library's kernels."""

    @staticmethod
    def forward(ctx, x, w1, w2, t):
        ws = mlp_step(x.detach(), w1.detach(), w2.detach(), t.detach())
        ctx.ws = ws
        return ws.loss[0].clone()

    @staticmethod
    def backward(ctx, grad):
        ws = ctx.ws
        g = grad.to(torch.float32)
        return ws.dx * g, ws.dw1 * g, ws.dw2 * g, None
