"""Leaf selection and mixed CPU / CIM inference: selected Conv2d and Linear
leaves of a CPU model run on the CUDA CIM runtime, the rest of the model on
CPU.

Mirrors python/cim22/layers.py of mlir-cim22 (discover_cim_layers,
validate_cim_layers and LayerOffload, :16-259) with the same arguments,
checks and error texts, for runtime="cuda": each selected leaf is compiled
in place through this package's torch.compile backend, receives its CPU
input, runs as CIM layers on one GPU and hands its CPU output back to the
outer model. The reference writes one compiled model library per layer under
artifact_dir; the CUDA runtime compiles in memory, so layer_artifacts stays
empty and artifact_dir is optional.
"""

from __future__ import annotations

import time
from collections.abc import Callable, Sequence
from functools import partial
from typing import Any, TypedDict

import torch

from .backend import backend
from .program import Program


class CimLayerInfo(TypedDict):
    """A selectable leaf module in a PyTorch model."""

    name: str
    type: str
    weight_shape: list[int]
    input_shape: list[int]
    output_shape: list[int]


def discover_cim_layers(model: torch.nn.Module,
                        example_inputs: tuple[torch.Tensor, ...] | None = None
                        ) -> list[CimLayerInfo]:
    """List the Conv2d/Linear leaves; optional example inputs run once to
    record their input and output shapes (forward hooks, removed afterwards
    even when the model raises). Running the model can change its state; the
    caller owns any reset (python/cim22/layers.py:26-63)."""
    found: list[CimLayerInfo] = []
    hooks = []

    def record(info: CimLayerInfo, _module, args, output) -> None:
        info["input_shape"] = list(args[0].shape)
        info["output_shape"] = list(output.shape)

    for name, module in model.named_modules(remove_duplicate=False):
        if not name or any(True for _ in module.children()):
            continue
        if not isinstance(module, (torch.nn.Conv2d, torch.nn.Linear)):
            continue
        info: CimLayerInfo = {"name": name, "type": type(module).__name__,
                              "weight_shape": list(module.weight.shape),
                              "input_shape": [], "output_shape": []}
        found.append(info)
        hooks.append(module.register_forward_hook(partial(record, info)))
    try:
        with torch.inference_mode():
            if example_inputs is not None:
                model(*example_inputs)
    finally:
        for hook in hooks:
            hook.remove()
    return found


def validate_cim_layers(model: torch.nn.Module, selected: Sequence[str] | None
                        ) -> tuple[str, ...]:
    """Exact, distinct, selectable leaf-module names (layers.py:66-103)."""
    if selected is None:
        return ()
    if isinstance(selected, str) or any(not isinstance(n, str) or not n for n in selected):
        raise ValueError("CIM layer names must be a sequence of non-empty strings")
    names = tuple(selected)
    if not names:
        raise ValueError("Select at least one CIM layer")
    if len(set(names)) != len(names):
        raise ValueError("CIM layer names must be unique")
    modules = dict(model.named_modules(remove_duplicate=False))
    aliases: dict[int, list[str]] = {}
    for name, module in modules.items():
        aliases.setdefault(id(module), []).append(name)
    for name in names:
        module = modules.get(name)
        if module is None:
            raise ValueError(f"Unknown CIM layer: {name}")
        if any(True for _ in module.children()):
            raise ValueError(f"CIM layer must be a leaf module: {name}")
        if not isinstance(module, (torch.nn.Conv2d, torch.nn.Linear)):
            raise ValueError(f"Unsupported CIM layer type: {name}")
        if len(aliases[id(module)]) > 1:
            raise ValueError(f"CIM layer has multiple names for the same module: {name}")
    return names


def _leaf_call(module: torch.nn.Module) -> Callable:
    """The leaf's call (hooks and forward) as a function of this package, so
    that Dynamo traces it: the reference compiles the leaf with
    module.compile(), but Dynamo skips the call frames of torch.nn's own
    modules when they are compiled directly, and LayerOffload selects exactly
    those (Conv2d, Linear). Installed as the module's compiled call, as
    module.compile() installs its own."""

    def call(*args, **kwargs):
        return module._call_impl(*args, **kwargs)

    return call


class LayerOffload:
    """Compile selected leaves in place and run the outer model on CPU.

    The model must be an evaluated CPU model with fixed weights and static
    input shapes. Construction compiles each selected layer for the CUDA
    runtime and warms it once under inference_mode with the example inputs;
    pass reset(model) for stateful networks (called after each warm-up).
    Each call returns the model's CPU outputs; an input that would compile a
    selected layer again is rejected, as in the reference
    (python/cim22/layers.py:106-259).
    """

    def __init__(self, model: torch.nn.Module, selected: Sequence[str],
                 example_inputs: tuple[torch.Tensor, ...], *, artifact_dir: Any = None,
                 runtime: str = "cuda", device: int = 0,
                 reset: Callable[[torch.nn.Module], None] | None = None) -> None:
        self.cim_layers = validate_cim_layers(model, selected)
        if not self.cim_layers:
            raise ValueError("Select at least one CIM layer")
        if runtime != "cuda":
            raise ValueError("Layer offload requires runtime='cuda'")
        if any(module.training for module in model.modules()):
            raise ValueError("Layer offload requires a model in eval mode")
        if any(value.device.type != "cpu"
               for value in (*model.parameters(), *model.buffers(), *example_inputs)):
            raise ValueError("Layer offload requires a CPU model and CPU inputs")
        self.model = model
        self.artifact_dir = artifact_dir
        self.layer_artifacts: dict[str, list[str]] = {}
        self.layer_compile_seconds: dict[str, float] = {}
        self._programs: dict[str, list[Program]] = {name: [] for name in self.cim_layers}
        compiled_calls = {}
        try:
            with torch.inference_mode():
                try:
                    for name, programs in self._programs.items():
                        module = model.get_submodule(name)
                        compiled_calls[module] = module._compiled_call_impl
                        started = time.perf_counter()
                        module._compiled_call_impl = torch.compile(
                            _leaf_call(module),
                            backend=partial(backend, _on_program=programs.append),
                            fullgraph=True, dynamic=False,
                            options={"runtime": runtime, "device": device})
                        if reset is not None:
                            reset(model)
                        previous = self._invocations()
                        model(*example_inputs)
                        if not programs:
                            raise RuntimeError(f"Missing runtime program for CIM layer: {name}")
                        self.layer_compile_seconds[name] = time.perf_counter() - started
                    self._dispatch_count = self._count_dispatches(previous)
                finally:
                    if reset is not None:
                        reset(model)
        except BaseException:
            for module, call in compiled_calls.items():
                module._compiled_call_impl = call
            raise

    def _invocations(self) -> dict[Program, int]:
        return {program: program.invocation_count
                for programs in self._programs.values() for program in programs}

    def _count_dispatches(self, previous: dict[Program, int]) -> int:
        total = 0
        for name, programs in self._programs.items():
            count = sum(program.cim_launch_count for program in programs
                        if program.invocation_count > previous.get(program, 0))
            if not count:
                raise RuntimeError(f"No CIM operations executed for layer: {name}")
            total += count
        return total

    @property
    def dispatch_count(self) -> int:
        """CIM layer kernels the selected layers ran in the latest call (the
        reference counts its tile dispatches here; the CUDA runtime runs each
        layer as whole-layer kernels)."""
        return self._dispatch_count

    def __call__(self, *inputs: torch.Tensor) -> Any:
        """Run the model; reject an input that compiled a selected layer again."""
        self._dispatch_count = 0
        previous = self._invocations()
        with torch.inference_mode():
            output = self.model(*inputs)
        if self._invocations().keys() != previous.keys():
            raise RuntimeError("Input triggered additional compilation; recompile the model")
        self._dispatch_count = self._count_dispatches(previous)
        return output
