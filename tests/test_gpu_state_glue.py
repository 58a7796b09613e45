"""Stateful elementwise glue through torch.compile runtime="cuda": the LIF
membrane loop, recurrence with Python state, and select_scatter, after the
reference's python/tests/test_backend.py:37-135,502-597. Every elementwise
step is one IEEE-rounded f32 operation, so results equal PyTorch CPU eager
bit for bit."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def reset_dynamo():
    torch._dynamo.reset()
    yield
    torch._dynamo.reset()


def compile_cuda(model):
    from cim22_b200 import backend

    name = backend.register()
    return torch.compile(model, backend=name, fullgraph=True, dynamic=False,
                         options={"runtime": "cuda"})


class LIF(torch.nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.register_buffer("voltage", (torch.arange(6, dtype=torch.float32) - 2) / 8)

    def forward(self, frames: torch.Tensor) -> torch.Tensor:
        spikes = torch.zeros_like(frames)
        voltage = self.voltage
        for step in range(frames.shape[0]):
            voltage = voltage + (frames[step] - voltage) / 2
            spike = (voltage >= 1).to(frames.dtype)
            voltage = (1 - spike) * voltage
            spikes[step] = spike
        self.voltage.copy_(voltage)
        return spikes


@pytest.mark.parametrize("steps", [3, 32])
def test_lif_frame_updates(steps):
    eager, model = LIF(), LIF()
    compiled = compile_cuda(model)
    frames = (torch.arange(steps * 6, dtype=torch.float32) % 15).reshape(steps, 6) / 8
    with torch.inference_mode():
        for value in (frames, frames + 0.25):
            got = compiled(value)
            want = eager(value)
            assert torch.equal(got, want)
            assert torch.equal(model.voltage, eager.voltage)
    assert model.voltage.abs().sum() > 0


def test_lif_random_frames_bitwise():
    rng = np.random.default_rng(1)
    eager, model = LIF(), LIF()
    compiled = compile_cuda(model)
    with torch.inference_mode():
        for _ in range(3):
            frames = torch.from_numpy(rng.standard_normal((16, 6)).astype(np.float32)) * 3
            got = compiled(frames)
            assert torch.equal(got, eager(frames))
            np.testing.assert_array_equal(model.voltage.numpy().view(np.uint32),
                                          eager.voltage.numpy().view(np.uint32))


class ResetSequence(torch.nn.Module):
    """Shared Linear with temporal recurrence and a plain Python reset state."""

    def __init__(self) -> None:
        super().__init__()
        self.linear = torch.nn.Linear(65, 17)
        self.v = 0.0
        with torch.no_grad():
            self.linear.weight.fill_(0.5)
            self.linear.bias.fill_(1.0)

    def reset(self) -> None:
        self.v = 0.0

    def forward(self, value: torch.Tensor) -> torch.Tensor:
        current = self.linear(value)
        if isinstance(self.v, float):
            self.v = torch.full_like(current[0].data, self.v)
        spikes = []
        for frame in current:
            self.v = (self.v + frame) * 0.5
            spike = (self.v >= 48.0).to(current.dtype)
            self.v = self.v * (1.0 - spike)
            spikes.append(spike)
        return torch.stack(spikes)


def test_reset_sequence():
    model = ResetSequence().eval()
    value = torch.full((2, 3, 65), 2.0)
    value[:, 1] *= 2
    value[:, 2] *= 0.5
    other_value = value * 2
    with torch.inference_mode():
        model(value)
        model.reset()
        compiled = compile_cuda(model)
        first = compiled(value)
        expected = torch.ones(2, 3, 17)
        expected[0, 0] = 0
        expected[:, 2] = 0
        assert torch.equal(first, expected)
        model.reset()
        second = compiled(other_value)
        expected_second = torch.ones_like(second)
        expected_second[0, 2] = 0
        assert torch.equal(second, expected_second)
        model.reset()
        assert torch.equal(compiled(value), first)


def test_select_scatter_keeps_old_values():
    def update(value):
        first = torch.select_scatter(value, value[:, 0], dim=-2, index=-1)
        second = torch.select_scatter(first, first[:, 1], dim=1, index=0)
        return first, second, value[:, -1]

    value = torch.arange(24, dtype=torch.float32).reshape(2, 3, 4)
    before = value.clone()
    compiled = compile_cuda(update)
    with torch.inference_mode():
        got = compiled(value)
        want = update(value)
    assert len(got) == 3
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert torch.equal(value, before)
