"""BASELINE config 3, the 2-layer MLP forward + backward, on the B200: against the reference's own `derive grad`
output (tests/golden/mlp_grad.npz: oracle/grad/mlp_grad.cairn built by the reference's compiler, its dense layers and
their adjoints chained with relu_grad, mse_grad and cr::fp::narrow), against the oracle's restatement of those loops
(oracle_mlp_step, pinned bit for bit to the same fixture by tests/test_oracle.py) at larger reduced shapes, and
against torch's own f32 autograd as a third reference. The bf16 intermediates (H, dY, dH) are stored as the
reference stores them; results agree within the north star's bf16 tolerance (Frobenius 2e-2), and in practice to
about 1e-3."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from cairn_b200 import mlp
from oracle import restated

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _rel(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).ravel()


def test_mlp_step_against_the_reference_derive_grad(cuda):
    """The device step on the fixture's operands against the reference's derive-grad chain: H within one bf16
    rounding plus the multiply's contract bound of the reference's f32 sums, element by element; the ReLU mask
    exactly where H > 0; every other tensor within Frobenius 2e-2; the loss within 1e-3."""
    d = np.load(GOLDEN / "mlp_grad.npz")
    B, D, H, O = map(int, d["shape"])
    x, w1, w2, t = d["x"], d["w1"], d["w2"], d["t"]
    dev = lambda bits, shape: torch.from_numpy(bits.view(np.int16).copy()).to(cuda).view(torch.bfloat16).view(shape)
    ws = mlp.mlp_step(dev(x, (B, D)), dev(w1, (D, H)), dev(w2, (H, O)), torch.from_numpy(t).to(cuda).view(B, O))
    cairn_b200.stream_status()
    want_h = inputs.decode("bf16", d["want/H"])
    got_h = inputs.decode("bf16", _bits(ws.h))
    mag = np.abs(inputs.decode("bf16", x).reshape(B, D)) @ np.abs(inputs.decode("bf16", w1).reshape(D, H))
    tol = 2.0**-8 * np.abs(want_h) + 2 * (D + 1) * 2.0**-22 * mag.ravel()
    assert (np.abs(got_h - want_h) <= tol).all()
    assert _rel(ws.y.cpu().numpy(), d["want/Y"]) < 2e-2
    assert _rel(inputs.decode("bf16", _bits(ws.dy)), inputs.decode("bf16", d["want/dY"])) < 2e-2
    for name in ("dW2", "dW1", "dX"):
        assert _rel(getattr(ws, name.lower()).cpu().numpy(), d[f"want/{name}"]) < 2e-2, name
    got_dh = inputs.decode("bf16", _bits(ws.dh))
    assert _rel(got_dh, inputs.decode("bf16", d["want/dH"])) < 2e-2
    assert (got_dh[got_h <= 0] == 0).all()
    want_loss = float(d["want/loss"][0])
    assert abs(float(ws.loss.item()) - want_loss) <= 1e-3 * abs(want_loss)


@pytest.mark.parametrize("B,D,H,O", [(128, 256, 512, 128), (264, 136, 392, 200), (512, 512, 1024, 512)])
def test_mlp_step_against_the_oracle(cuda, B, D, H, O):
    rng = np.random.default_rng(B + D)
    x = inputs.encode("bf16", rng.standard_normal(B * D))
    w1 = inputs.encode("bf16", rng.standard_normal(D * H) * 0.02 * 16)
    w2 = inputs.encode("bf16", rng.standard_normal(H * O) * 0.02 * 16)
    t = rng.standard_normal(B * O).astype(np.float32)
    want = restated.mlp_step(x, w1, w2, t, B, D, H, O)
    dev = lambda bits, shape: torch.from_numpy(bits.view(np.int16).copy()).to(cuda).view(torch.bfloat16).view(shape)
    ws = mlp.mlp_step(dev(x, (B, D)), dev(w1, (D, H)), dev(w2, (H, O)), torch.from_numpy(t).to(cuda).view(B, O))
    cairn_b200.stream_status()
    got_h = inputs.decode("bf16", _bits(ws.h))
    assert _rel(got_h, inputs.decode("bf16", want["H"])) < 1e-2
    assert _rel(ws.y.cpu().numpy(), want["Y"]) < 1e-2
    assert abs(float(ws.loss.item()) - float(want["loss"][0])) <= 1e-3 * abs(float(want["loss"][0]))
    for name in ("dW2", "dW1", "dX"):
        assert _rel(getattr(ws, name.lower()).cpu().numpy(), want[name]) < 2e-2, name
    assert _rel(inputs.decode("bf16", _bits(ws.dh)), inputs.decode("bf16", want["dH"])) < 2e-2
    # the ReLU mask is exactly where H > 0
    assert (inputs.decode("bf16", _bits(ws.dh))[got_h <= 0] == 0).all()


def test_autograd_backward_runs_the_library_and_matches_torch(cuda):
    B, D, H, O = 256, 256, 512, 256
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(B, D, device=cuda, generator=g).bfloat16()
    w1 = (torch.randn(D, H, device=cuda, generator=g) * 0.05).bfloat16().requires_grad_()
    w2 = (torch.randn(H, O, device=cuda, generator=g) * 0.05).bfloat16().requires_grad_()
    xr = x.clone().requires_grad_()
    t = torch.randn(B, O, device=cuda, generator=g)
    loss = mlp.MLPLoss.apply(xr, w1, w2, t)
    loss.backward()
    cairn_b200.stream_status()
    # torch's own f32 autograd on the same bf16 values
    X, W1, W2 = (v.detach().float().requires_grad_() for v in (x, w1, w2))
    ref = ((torch.relu(X @ W1) @ W2 - t) ** 2).mean()
    ref.backward()
    assert abs(loss.item() - ref.item()) <= 1e-2 * ref.item()
    for got, want in ((xr.grad, X.grad), (w1.grad, W1.grad), (w2.grad, W2.grad)):
        assert _rel(got.float().cpu().numpy(), want.cpu().numpy()) < 2e-2


def test_steps_fed_from_host_memory_match_steps_on_device_copies(cuda):
    """mlp.step_from_host: batches copied in on the feed's stream while the step before computes, the loss copied
    back; every step's loss and gradients equal, bit for bit, those of the same step run from device tensors."""
    B, D, Hd, O = 512, 256, 1024, 512
    g = torch.Generator(device=cuda).manual_seed(3)
    w1 = (torch.randn(D, Hd, device=cuda, generator=g) * 0.02).bfloat16()
    w2 = (torch.randn(Hd, O, device=cuda, generator=g) * 0.02).bfloat16()
    batches = [(torch.randn(B, D, device=cuda, generator=g).bfloat16(), torch.randn(B, O, device=cuda, generator=g))
               for _ in range(3)]
    want = []
    for x, t in batches:
        ws = mlp.mlp_step(x, w1, w2, t)
        want.append((ws.loss.clone(), ws.dw1.clone(), ws.dw2.clone(), ws.dx.clone()))
    host = [(x.cpu().pin_memory(), t.cpu().pin_memory()) for x, t in batches]
    feed = mlp.HostFeed(B, D, O, cuda)
    ws = mlp.MLPWorkspace(B, D, Hd, O, cuda)
    losses = [torch.empty(1, dtype=torch.float32).pin_memory() for _ in range(5)]
    stream = torch.cuda.current_stream(cuda)
    for i in range(5):
        x_h, t_h = host[i % 3]
        mlp.step_from_host(feed, x_h, t_h, w1, w2, ws, losses[i], stream)
        if i == 4:
            torch.cuda.synchronize()
            w_loss, w_dw1, w_dw2, w_dx = want[i % 3]
            assert torch.equal(ws.dw1, w_dw1) and torch.equal(ws.dw2, w_dw2) and torch.equal(ws.dx, w_dx)
    torch.cuda.synchronize()
    cairn_b200.stream_status()
    for i in range(5):
        assert losses[i].item() == want[i % 3][0].item(), i
