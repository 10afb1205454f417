"""``AttributionTask``: what to attribute -- a model, the loss whose gradients are compared
(and optionally a different target for the query side), and the checkpoints to attribute at.

A model wrapped in DDP or FSDP can be handed over as is: the capture hooks are put on the
module inside the wrapper, while forward passes go through the wrapper so that its
collectives run.  :meth:`AttributionTask.from_dattri` adapts a task of the ``dattri``
package, whose losses take a parameter dictionary.  Public names and constructor keywords
as in the reference (``dattri_llm/task.py``).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from pathlib import Path

import torch
from torch import nn

LossFunc = Callable[[nn.Module, object], torch.Tensor]


def default_loss_func(model: nn.Module, batch: object) -> torch.Tensor:
    """The loss a Hugging Face style model returns for a keyword batch: ``model(**batch).loss``.

    Raises:
        TypeError: *batch* is not a mapping of model keywords.
        ValueError: the model output carries no ``loss`` (e.g. no labels in the batch).
    """
    if not isinstance(batch, dict):
        raise TypeError(f"default_loss_func calls model(**batch) and needs a dict batch, got "
                        f"{type(batch).__name__}; give the task a loss_func for this batch type.")
    out = model(**batch)
    loss = getattr(out, "loss", None)
    if loss is None:
        raise ValueError(f"{type(out).__name__} from model(**batch) has no loss (are labels missing "
                         "from the batch?); give the task a loss_func.")
    return loss


def _wrapper_types() -> tuple[type, ...]:
    from torch.nn.parallel import DistributedDataParallel

    found: list[type] = [DistributedDataParallel]
    try:
        from torch.distributed.fsdp import FullyShardedDataParallel

        found.append(FullyShardedDataParallel)
    except ImportError:  # pragma: no cover - builds without distributed support
        pass
    return tuple(found)


def default_checkpoint_load_func(model: nn.Module, checkpoint: object) -> nn.Module:
    """Load *checkpoint* -- a state dict, a path to a saved one, or ``None`` for "keep the
    current parameters" -- into *model* and return it."""
    if checkpoint is None:
        return model
    if isinstance(checkpoint, (str, Path)):
        where = next(iter(model.parameters())).device
        checkpoint = torch.load(checkpoint, map_location=where, weights_only=True)
    model.load_state_dict(checkpoint)
    return model


@dataclass
class _Model:
    """The module the hooks see (``inner``) and the one forwards run through (``outer``;
    the same object unless the model came wrapped)."""

    inner: nn.Module
    outer: nn.Module

    @classmethod
    def of(cls, model: nn.Module) -> _Model:
        return cls(model.module if isinstance(model, _wrapper_types()) else model, model)

    @property
    def wrapped(self) -> bool:
        return self.outer is not self.inner


class AttributionTask:
    """A model, the loss (and query target) to attribute, and the checkpoints to visit.

    Args:
        loss_func: ``loss_func(model, batch) -> scalar`` for the training side;
            ``None`` uses :func:`default_loss_func`.
        model: the model, optionally wrapped in DDP / FSDP.
        checkpoints: one checkpoint or a sequence of them (state dicts, paths, or ``None``
            for the parameters the model holds).
        target_func: the query side's function (defaults to *loss_func*).
        checkpoints_load_func: ``load(model, checkpoint) -> model`` replacing
            :func:`default_checkpoint_load_func`.
    """

    def __init__(self, loss_func: LossFunc | None, model: nn.Module, checkpoints: object = None,
                 target_func: LossFunc | None = None, checkpoints_load_func: Callable | None = None) -> None:
        self.loss_func: LossFunc = loss_func or default_loss_func
        self.target_func: LossFunc = target_func or self.loss_func
        self._handle = _Model.of(model)
        self.checkpoints: list = (list(checkpoints) if isinstance(checkpoints, Sequence)
                                  and not isinstance(checkpoints, (str, bytes)) else [checkpoints])
        if len(self.checkpoints) == 0:
            raise ValueError("an AttributionTask needs at least one checkpoint (None = the current parameters).")
        self._loader = checkpoints_load_func or default_checkpoint_load_func
        if (self._loader is default_checkpoint_load_func and self._handle.wrapped
                and any(ck is not None for ck in self.checkpoints)):
            raise ValueError("the default checkpoint loader writes a plain state dict, which a DDP/FSDP "
                             "wrapper's module does not accept; use checkpoints=None (attribute at the "
                             "wrapper's parameters) or a checkpoints_load_func that loads through the wrapper.")
        self.current_checkpoint_idx: int | None = None

    # ------------------------------------------------------------------ models
    @property
    def model(self) -> nn.Module:
        """The module the capture hooks attach to (inside any wrapper)."""
        return self._handle.inner

    @property
    def forward_model(self) -> nn.Module | None:
        """The DDP / FSDP wrapper forwards must run through, or ``None`` for a plain model."""
        return self._handle.outer if self._handle.wrapped else None

    @property
    def is_wrapped(self) -> bool:
        """Whether the model came inside a DDP / FSDP wrapper."""
        return self._handle.wrapped

    def get_model(self) -> nn.Module:
        """Same as :attr:`model`."""
        return self._handle.inner

    # ------------------------------------------------------------------ checkpoints
    def get_checkpoints(self) -> list:
        """The checkpoints, in visiting order."""
        return self.checkpoints

    def num_checkpoints(self) -> int:
        """How many checkpoints the task visits."""
        return len(self.checkpoints)

    def load_checkpoint(self, index: int) -> nn.Module:
        """Make checkpoint *index* the model's parameters (skipped when it already is) and
        return the hooked module.

        Raises:
            ValueError: the loader replaced a wrapped model's module instead of loading in place.
        """
        if index == self.current_checkpoint_idx:
            return self._handle.inner
        result = self._loader(self._handle.inner, self.checkpoints[index])
        if result is not self._handle.inner:
            if self._handle.wrapped:
                raise ValueError("checkpoints_load_func must load a wrapped model in place and return the "
                                 "module it was given; it returned a different module.")
            self._handle = _Model(result, result)
        self.current_checkpoint_idx = index
        return self._handle.inner

    def invalidate_checkpoint(self) -> None:
        """Mark the parameters as changed in place (e.g. trained by a trajectory run): the
        next :meth:`load_checkpoint` loads even the index loaded last."""
        self.current_checkpoint_idx = None

    # ------------------------------------------------------------------ dattri interop
    @classmethod
    def from_dattri(cls, task: object) -> AttributionTask:
        """This class's task for a ``dattri`` ``AttributionTask`` (an instance of this class
        passes through unchanged).

        Raises:
            TypeError: *task* does not look like a dattri task.
        """
        if isinstance(task, cls):
            return task
        needed = ("original_loss_func", "original_target_func", "model", "checkpoints")
        missing = [name for name in needed if not hasattr(task, name)]
        if missing:
            raise TypeError(f"not a dattri AttributionTask: it has no {missing}.")
        return cls(_on_named_parameters(task.original_loss_func), task.model, checkpoints=list(task.checkpoints),
                   target_func=_on_named_parameters(task.original_target_func),
                   checkpoints_load_func=task.checkpoints_load_func)


def _on_named_parameters(func: Callable) -> LossFunc:
    """A ``(model, batch)`` loss from dattri's functional ``(params_dict, batch)`` form."""
    return lambda model, batch: func(dict(model.named_parameters()), batch)


def as_task(task: object) -> AttributionTask:
    """Coerce *task* with :meth:`AttributionTask.from_dattri`."""
    return AttributionTask.from_dattri(task)
