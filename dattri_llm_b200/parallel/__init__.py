"""Multi-GPU machinery: process-group helpers, DDP/FSDP wrapping and the fused
compute + collective paths over NVLink (symmetric-memory peer access)."""
