from .kernel_deltanet_layer import KernelDeltaNetLayer, KernelTTTLayer

__all__ = ["KernelDeltaNetLayer", "KernelTTTLayer"]
