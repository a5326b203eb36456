"""dsv4_plugin.models — the MoE layer that replaces vLLM's DeepSeek-V4 MoE."""

from dsv4_plugin.models.deepseek_v4 import OffloadDeepseekV4MoE, install_patches

__all__ = ["OffloadDeepseekV4MoE", "install_patches"]
