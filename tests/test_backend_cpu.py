"""torch.compile backend behaviour that needs no GPU: options, reference
mode, grad rejection and identity guards on frozen module inputs."""

import pytest
import torch

from cim22_b200 import backend, workloads


def test_reference_runtime_is_plain_cpu_pytorch():
    name = backend.register()
    assert backend.register() == name
    model, x = workloads.build("lenet", 2)
    compiled = torch.compile(model, backend=name, fullgraph=True, dynamic=False,
                             options={"runtime": "reference"})
    with torch.inference_mode():
        assert torch.equal(compiled(x), model(x))


def test_rejects_unknown_runtime_and_grad():
    with pytest.raises(ValueError, match="runtime"):
        backend._validate({"runtime": "usb"})
    with pytest.raises(ValueError, match="sign-split"):
        backend._validate({"bf16_compensation": "exact"})
    for mode in ("sign-split", "legacy", "none"):
        backend._validate({"bf16_compensation": mode})
    gm = torch.fx.symbolic_trace(torch.nn.ReLU())
    with torch.enable_grad(), pytest.raises(ValueError, match="no_grad"):
        backend.backend(gm, [torch.ones(2)], options={"runtime": "cuda"})


def test_frozen_parameters_are_identity_guarded(monkeypatch):
    """A second module of the same class must recompile, not reuse the first
    module's frozen weights (python/cim22/backend.py:207-210)."""

    class FakeProgram:
        def __init__(self, gm, example, frozen, device, name, bf16_compensation, chain):
            self.gm, self.example, self.frozen = gm, example, frozen

        def capture(self):
            pass

        def __call__(self, *values):
            it = iter(values)
            args = [e if i in self.frozen else next(it) for i, e in enumerate(self.example)]
            return self.gm(*args)

    monkeypatch.setattr(backend, "Program", FakeProgram)
    name = backend.register()

    class M(torch.nn.Module):
        def __init__(self, v):
            super().__init__()
            self.w = torch.nn.Parameter(torch.full((4, 4), float(v)), requires_grad=False)

        def forward(self, x):
            return x @ self.w

    x = torch.ones(2, 4)
    with torch.inference_mode():
        for v in (1.0, 2.0, 3.0):
            m = M(v)
            c = torch.compile(m, backend=name, options={"runtime": "cuda"})
            assert torch.equal(c(x), x @ m.w)
