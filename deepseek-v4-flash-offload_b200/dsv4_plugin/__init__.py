"""dsv4_plugin — B200 (sm_100a) routed-expert MoE for DeepSeek-V4-Flash.

vLLM plugin entry point (``[project.entry-points."vllm.general_plugins"]
dsv4_offload = "dsv4_plugin:register_model"``), same name and behaviour as
the reference plugin (dsv4_plugin/__init__.py:18-19): ``register_model()``
idempotently installs ``OffloadDeepseekV4MoE`` and the ``load_weights`` tee.
"""

__all__ = ["register_model"]


def register_model():
    from dsv4_plugin.models.deepseek_v4 import install_patches

    install_patches()
