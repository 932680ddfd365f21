"""Drop-in installation of the fused ops into transformers Qwen3 models."""

from .qwen3 import (AttentionBackend, FusedDecodeAttention, ReferenceAttention,
                    allocate_kv_cache, batch_mapping, forget_batch_mapping,
                    fused_qwen3_model_loader, install_fused, install_operator_overrides,
                    restore_operator_overrides)

__all__ = ["AttentionBackend", "FusedDecodeAttention", "ReferenceAttention", "allocate_kv_cache",
           "batch_mapping", "forget_batch_mapping", "fused_qwen3_model_loader", "install_fused",
           "install_operator_overrides", "restore_operator_overrides"]
