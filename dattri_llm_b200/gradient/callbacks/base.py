"""Base class of :class:`HookManager` callbacks (the extension point of the capture engine).

Callbacks see every layer's forward and backward fire, each completed step's
:class:`GradientRecord` (dispatched outside the manager's lock, so a callback may
run a secondary forward/backward through the same hooks) and the end of the
``collect()`` context.  Parity: reference ``dattri_llm/gradient/callbacks/base.py``.
"""

from __future__ import annotations


class HookManagerCallback:
    """No-op hooks; override what you need (``on_register(manager)`` is optional)."""

    def on_layer_forward(self, layer_name: str, activation, layer_type: str,
                         module_kwargs: dict | None) -> None:
        """A hooked layer ran forward (*activation* projected for pre-projected layers)."""

    def on_layer_backward(self, layer_name: str, grad_output, layer_type: str,
                          module_kwargs: dict | None) -> None:
        """A hooked layer received its output gradient."""

    def on_step_end(self, record) -> None:
        """A backward completed and its record was assembled."""

    def on_context_end(self) -> None:
        """The ``collect()`` context exited."""
