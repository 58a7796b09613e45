"""torch.compile backend ``cim22`` with the CUDA execution runtime.

Mirrors the reference's backend (python/cim22/backend.py:102-235 of mlir-cim22)
and its options (python/cim22/compiler.py:28-93):

  runtime="cuda"       new: lower the captured graph to CIM layers and glue
                       kernels on a B200 (this package);
  runtime="reference"  the captured graph with CPU PyTorch operators, exactly as
                       the reference's reference mode.
  chain                "auto" (default): a network that is one chain of Conv2d /
                       Linear layers with ReLU/GELU and 2x2 max pools runs either
                       as one fused persistent kernel or layer by layer, whichever
                       a timed launch finds faster (same bits); True / False force
                       one of them.

Read-only module parameters and buffers are frozen into the compiled program,
as the reference freezes them (backend.py:161-196); Dynamo guards on their
identity. Gradients must be disabled. bf16_compensation selects "sign-split"
(the default), or the reference's diagnostic "legacy" and "none" modes
(compiler.py:25,34-36).
Inputs may be CPU or CUDA tensors; outputs are returned on the inputs' device.
"""

from __future__ import annotations

from typing import Any, Callable, Sequence, TypedDict

import torch

from .program import Program


class BackendOptions(TypedDict, total=False):
    runtime: str
    bf16_compensation: str
    device: int
    cuda_graph: bool
    chain: Any  # "auto" (default), True or False: the fused layer chain lowering
    artifact_dir: Any
    debug_dir: Any


def _validate(options: dict) -> None:
    runtime = options.get("runtime", "cuda")
    if runtime not in ("cuda", "reference"):
        raise ValueError("CIM22 runtime must be one of ('reference', 'cuda') in this backend")
    if options.get("bf16_compensation", "sign-split") not in ("sign-split", "legacy", "none"):
        raise ValueError(
            "CIM22 bf16_compensation must be 'sign-split', 'legacy' or 'none'")
    if options.get("usb_config") is not None or options.get("usb_session") is not None:
        raise ValueError("CIM22 usb options require runtime='usb'")


def _is_module_input(node: torch.fx.Node) -> bool:
    grapharg = node.meta.get("grapharg")
    if grapharg is None:
        return False
    from torch._dynamo.source import NNModuleSource, UnspecializedParamBufferSource

    source = grapharg.source
    while source is not None:
        if isinstance(source, (NNModuleSource, UnspecializedParamBufferSource)):
            return True
        source = getattr(source, "base", None)
    name = getattr(grapharg.source, "name", lambda: "")
    text = name() if callable(name) else str(name)
    return "_modules_" in text or "_parameters_" in text or "_buffers_" in text


def _is_mutated(node: torch.fx.Node) -> bool:
    import operator

    from .program import MUTATING_METHODS

    for user in node.users:
        if user.args and user.args[0] is node and (
                (user.op == "call_method" and user.target in MUTATING_METHODS) or
                (user.op == "call_function" and user.target is operator.setitem)):
            return True
    return False


def backend(gm: torch.fx.GraphModule, example_inputs: Sequence[torch.Tensor], *,
            options: BackendOptions | None = None,
            _on_program: Callable[[Program], None] | None = None) -> Callable:
    """Compile a static inference graph for torch.compile. _on_program receives
    each compiled program (LayerOffload tracks its layers' programs with it, as
    the reference's backend hands out sessions through _on_session)."""
    options = dict(options or {})
    _validate(options)
    if torch.is_grad_enabled():
        raise ValueError("Use torch.no_grad() or torch.inference_mode() with CIM22")
    runtime = options.get("runtime", "cuda")
    if runtime == "reference":
        if any(isinstance(v, torch.Tensor) and v.device.type != "cpu" for v in example_inputs):
            raise ValueError("CIM22 reference requires CPU tensors")
        return gm.forward
    placeholders = list(gm.graph.find_nodes(op="placeholder"))
    # Module state the forward writes (a LIF membrane buffer updated with
    # copy_ or slice writes) stays a runtime input and is written back after
    # each call, as the reference keeps mutated inputs out of its frozen set
    # (python/cim22/backend.py:171-185).
    mutated = {i for i, node in enumerate(placeholders) if _is_mutated(node)}
    frozen = {i for i, node in enumerate(placeholders)
              if isinstance(example_inputs[i], torch.Tensor) and _is_module_input(node)
              and i not in mutated}
    # Frozen values cannot serve another module's parameters or buffers: guard
    # on their identity so Dynamo recompiles for a different module
    # (python/cim22/backend.py:207-210 of the reference does the same).
    from torch._dynamo.guards import GuardBuilder, install_guard

    for i in frozen:
        grapharg = placeholders[i].meta.get("grapharg")
        if grapharg is None or grapharg.source is None:
            raise ValueError("CIM22 cannot guard a frozen module input without a source")
        install_guard(grapharg.source.make_guard(GuardBuilder.ID_MATCH))
    device = int(options.get("device", 0))
    program = Program(gm, [e.detach() if isinstance(e, torch.Tensor) else e
                           for e in example_inputs],
                      frozen=frozen, device=device, name="cim22_cuda",
                      bf16_compensation=options.get("bf16_compensation", "sign-split"),
                      chain=options.get("chain", "auto"))
    if options.get("cuda_graph", True):
        program.capture()
    if _on_program is not None:
        _on_program(program)
    inputs = [i for i in range(len(placeholders)) if i not in frozen]

    def run(*values):
        result = program(*(values[i] for i in inputs))
        return result if isinstance(result, tuple) else (result,)

    run.program = program  # type: ignore[attr-defined]
    return run


_registered: str | None = None


def register(name: str = "cim22") -> str:
    """Register the backend with Dynamo, as ``name`` unless another backend
    already holds it (then as ``cim22_cuda``). Idempotent; returns the name."""
    global _registered
    if _registered is not None:
        return _registered
    from torch._dynamo import list_backends, register_backend

    def cim22(gm, example_inputs, options=None):
        return backend(gm, example_inputs, options=options)

    if name in list_backends(exclude_tags=()):
        name = "cim22_cuda"
    register_backend(name=name)(cim22)
    _registered = name
    return name
