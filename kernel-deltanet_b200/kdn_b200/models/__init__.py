from .kernel_deltanet_lm import HybridCache, KernelDeltaNetLM, KernelTTTLM

__all__ = ["HybridCache", "KernelDeltaNetLM", "KernelTTTLM"]
