"""``AttributionTask``: a model, the loss to attribute (and an optional separate
target), and the checkpoints to attribute at.

Parity: reference ``dattri_llm/task.py:42-251``.  A DDP/FSDP-wrapped model can be
passed directly: hooks go on the unwrapped module, the forward runs through the
wrapper.  ``from_dattri`` adapts a dattri ``AttributionTask`` (functional losses
taking a parameter dict).
"""

from __future__ import annotations

from collections.abc import Callable
from pathlib import Path

import torch
from torch import nn


def default_loss_func(model: nn.Module, batch: object) -> torch.Tensor:
    """``model(**batch).loss``.

    Raises:
        TypeError / ValueError: for a non-dict batch or an output without ``.loss``.
    """
    if not isinstance(batch, dict):
        raise TypeError("default_loss_func expects a dict batch (model(**batch).loss); pass a "
                        "loss_func for other batch formats.")
    loss = getattr(model(**batch), "loss", None)
    if loss is None:
        raise ValueError("model(**batch) returned no .loss; pass a loss_func that computes the loss "
                         "from the model output (e.g. with labels).")
    return loss


def _unwrap(model: nn.Module) -> nn.Module:
    from torch.nn.parallel import DistributedDataParallel

    wrappers: tuple[type, ...] = (DistributedDataParallel,)
    try:
        from torch.distributed.fsdp import FullyShardedDataParallel

        wrappers = (*wrappers, FullyShardedDataParallel)
    except ImportError:  # pragma: no cover
        pass
    return model.module if isinstance(model, wrappers) else model


def default_checkpoint_load_func(model: nn.Module, checkpoint: object) -> nn.Module:
    """Load a state dict (or a path to one) into *model*; ``None`` keeps the parameters."""
    if checkpoint is None:
        return model
    if isinstance(checkpoint, (str, Path)):
        checkpoint = torch.load(checkpoint, map_location=next(model.parameters()).device, weights_only=True)
    model.load_state_dict(checkpoint)
    return model


class AttributionTask:
    """A model, its loss (and target), and the checkpoints to attribute at."""

    def __init__(self, loss_func: Callable | None, model: nn.Module, checkpoints: object = None,
                 target_func: Callable | None = None, checkpoints_load_func: Callable | None = None) -> None:
        self.loss_func = loss_func if loss_func is not None else default_loss_func
        self.target_func = target_func if target_func is not None else self.loss_func
        self._forward_model = model
        self._model = _unwrap(model)
        self.checkpoints = list(checkpoints) if isinstance(checkpoints, (list, tuple)) else [checkpoints]
        if not self.checkpoints:
            raise ValueError("checkpoints must hold at least one checkpoint.")
        self._load = checkpoints_load_func or default_checkpoint_load_func
        if (self._load is default_checkpoint_load_func and self.is_wrapped
                and any(c is not None for c in self.checkpoints)):
            raise ValueError("The default checkpoint loader cannot load a state dict into a DDP/FSDP-wrapped "
                             "model; pass checkpoints=None to attribute at the parameters it holds, or a "
                             "checkpoints_load_func that loads through the wrapper.")
        self.current_checkpoint_idx: int | None = None

    @property
    def model(self) -> nn.Module:
        """The unwrapped model (hooks go here)."""
        return self._model

    @property
    def forward_model(self) -> nn.Module | None:
        """The DDP/FSDP wrapper the task came in, else ``None``."""
        return self._forward_model if self.is_wrapped else None

    @property
    def is_wrapped(self) -> bool:
        """Whether the model came wrapped."""
        return self._forward_model is not self._model

    def get_model(self) -> nn.Module:
        """The unwrapped model."""
        return self._model

    def get_checkpoints(self) -> list:
        """The checkpoints."""
        return self.checkpoints

    def num_checkpoints(self) -> int:
        """Number of checkpoints."""
        return len(self.checkpoints)

    def load_checkpoint(self, index: int) -> nn.Module:
        """Load checkpoint *index* (no-op when already loaded) and return the model.

        Raises:
            ValueError: when a loader returns a new module for a wrapped model.
        """
        if self.current_checkpoint_idx != index:
            loaded = self._load(self._model, self.checkpoints[index])
            if loaded is not self._model:
                if self.is_wrapped:
                    raise ValueError("checkpoints_load_func returned a new module for a wrapped model; it "
                                     "must load in place through the wrapper and return the same module.")
                self._model = self._forward_model = loaded
            self.current_checkpoint_idx = index
        return self._model

    def invalidate_checkpoint(self) -> None:
        """Forget which checkpoint is loaded: the parameters were changed in place (a
        trajectory run trained them), so the next :meth:`load_checkpoint` reloads."""
        self.current_checkpoint_idx = None

    @classmethod
    def from_dattri(cls, task: object) -> AttributionTask:
        """Adapt a dattri ``AttributionTask`` (or return an instance of this class as is).

        Raises:
            TypeError: when *task* lacks dattri's attributes.
        """
        if isinstance(task, cls):
            return task
        for attr in ("original_loss_func", "original_target_func", "model", "checkpoints"):
            if not hasattr(task, attr):
                raise TypeError(f"from_dattri expects a dattri AttributionTask (missing {attr!r}).")
        return cls(_functional(task.original_loss_func), task.model, checkpoints=list(task.checkpoints),
                   target_func=_functional(task.original_target_func),
                   checkpoints_load_func=task.checkpoints_load_func)


def _functional(func: Callable) -> Callable:
    def loss_fn(model: nn.Module, batch: object) -> torch.Tensor:
        return func(dict(model.named_parameters()), batch)
    return loss_fn


def as_task(task: object) -> AttributionTask:
    """:meth:`AttributionTask.from_dattri`."""
    return AttributionTask.from_dattri(task)
