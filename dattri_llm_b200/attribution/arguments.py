"""``AttributionArguments``: the HF-TrainingArguments-like run configuration.

Field names, defaults and validation match the reference's
(``dattri_llm/attribution/arguments.py:44-625``) so a configuration written for
either framework runs on the other; ``LOCAL_RANK`` / ``WORLD_SIZE`` / ``RANK`` come
from the environment the launcher (``torchrun``) sets.  B200 additions are
``cuda_graphs`` (capture the frozen probe's step once and replay it) and
``capture_stream`` (not the default) -- see :class:`GradientStreamer`.
"""

from __future__ import annotations

import json
import logging
import os
from dataclasses import dataclass, field
from functools import cached_property
from pathlib import Path

import torch

logger = logging.getLogger(__name__)
_DICT_FIELDS = ("gradient_checkpointing_kwargs", "fsdp_config", "deepspeed")


@dataclass
class AttributionArguments:
    """Configuration for running a training-data attribution algorithm."""

    output_dir: str
    per_device_train_batch_size: int = 8
    per_device_eval_batch_size: int = 8
    learning_rate: float = 5e-5
    weight_decay: float = 0.0
    optim: str = "adamw_torch"
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    adam_epsilon: float = 1e-8
    lr_scheduler_type: str = "linear"
    warmup_steps: int = 0
    gradient_accumulation_steps: int = 1
    max_grad_norm: float | None = 1.0
    gradient_checkpointing: bool = False
    gradient_checkpointing_kwargs: dict | str | None = None
    use_cpu: bool = False
    bf16: bool = False
    fp16: bool = False
    tf32: bool | None = None
    seed: int = 42
    data_seed: int | None = None
    full_determinism: bool = False
    dataloader_num_workers: int = 0
    dataloader_pin_memory: bool = True
    dataloader_persistent_workers: bool = False
    dataloader_prefetch_factor: int | None = None
    async_disk_write: bool = False
    recompute_gradients: bool = False
    ddp_find_unused_parameters: bool | None = None
    fsdp: str | list[str] = ""
    fsdp_config: dict | str | None = None
    deepspeed: dict | str | None = None
    cuda_graphs: bool = field(default=False, metadata={
        "help": "Frozen probes on CUDA: capture one forward+backward+capture step in a CUDA graph "
                "per batch shape and replay it (inputs copied into static buffers)."})

    def __post_init__(self) -> None:
        self.output_dir = str(Path(self.output_dir).expanduser())
        for name in _DICT_FIELDS:
            value = getattr(self, name)
            if isinstance(value, str):
                if value.startswith("{"):
                    setattr(self, name, json.loads(value))
                elif Path(value).is_file():
                    setattr(self, name, json.loads(Path(value).read_text(encoding="utf-8")))
        if self.data_seed is None:
            self.data_seed = self.seed
        if self.dataloader_pin_memory and not torch.cuda.is_available():
            self.dataloader_pin_memory = False
        if self.tf32 is not None:
            if torch.cuda.is_available():
                torch.backends.cuda.matmul.allow_tf32 = self.tf32
                torch.backends.cudnn.allow_tf32 = self.tf32
            else:
                logger.warning("tf32 has no effect without a CUDA device.")
        self._validate()

    def _validate(self) -> None:
        if self.bf16 and self.fp16:
            raise ValueError("bf16 and fp16 cannot both be True.")
        if self.per_device_train_batch_size <= 0:
            raise ValueError(f"per_device_train_batch_size must be > 0, got {self.per_device_train_batch_size}.")
        if self.per_device_eval_batch_size <= 0:
            raise ValueError(f"per_device_eval_batch_size must be > 0, got {self.per_device_eval_batch_size}.")
        if self.gradient_accumulation_steps < 1:
            raise ValueError(f"gradient_accumulation_steps must be >= 1, got {self.gradient_accumulation_steps}.")
        if self.max_grad_norm is not None and self.max_grad_norm <= 0:
            raise ValueError(f"max_grad_norm must be > 0 or None, got {self.max_grad_norm}.")
        if self.dataloader_prefetch_factor is not None and self.dataloader_prefetch_factor <= 0:
            raise ValueError(f"dataloader_prefetch_factor must be > 0 or None, got {self.dataloader_prefetch_factor}.")
        if self.dataloader_persistent_workers and self.dataloader_num_workers == 0:
            logger.warning("dataloader_persistent_workers=True has no effect when dataloader_num_workers=0.")

    @cached_property
    def _device_and_n_gpu(self) -> tuple[torch.device, int]:
        if self.use_cpu or not torch.cuda.is_available():
            return torch.device("cpu"), 0
        local = int(os.environ.get("LOCAL_RANK", "-1"))
        if local != -1:
            return torch.device("cuda", local), 1
        return torch.device("cuda"), torch.cuda.device_count()

    @property
    def device(self) -> torch.device:
        """The device this process computes on."""
        return self._device_and_n_gpu[0]

    @property
    def n_gpu(self) -> int:
        """GPUs this process drives."""
        return self._device_and_n_gpu[1]

    @property
    def world_size(self) -> int:
        """``WORLD_SIZE`` (1 outside a launcher)."""
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        return ws if ws > 0 else 1

    @property
    def process_index(self) -> int:
        """``RANK``."""
        return int(os.environ.get("RANK", "0"))

    @property
    def local_process_index(self) -> int:
        """``LOCAL_RANK``."""
        return int(os.environ.get("LOCAL_RANK", "0"))

    @property
    def train_batch_size(self) -> int:
        """Per-process train batch times the GPUs this process drives."""
        return self.per_device_train_batch_size * max(1, self.n_gpu)

    @property
    def eval_batch_size(self) -> int:
        """Per-process eval batch times the GPUs this process drives."""
        return self.per_device_eval_batch_size * max(1, self.n_gpu)

    @property
    def should_log(self) -> bool:
        """Rank 0 logs."""
        return self.process_index == 0

    @property
    def output_path(self) -> Path:
        """``output_dir`` as a path."""
        return Path(self.output_dir)
