"""Shared small configurations for tests."""
from packmla.config import ModelConfig


def small_gpu_config(**kw) -> ModelConfig:
    """Smallest config the MXFP4 kernels accept (hidden and intermediate multiples of 1024)."""
    base = dict(name="small", vocab_size=1000, hidden_size=1024, num_layers=4, num_heads=16, q_lora_rank=256,
                o_groups=4, o_lora_rank=256, compress_ratios=[0, 4, 128, 4], index_heads=8, index_dim=128,
                index_topk=32, n_routed_experts=8, moe_topk=2, moe_intermediate=1024, expert_format="mxfp4",
                dense_format="bf16", max_position=8192)
    base.update(kw)
    return ModelConfig(**base)
