from .ragged import ragged_prefill
from .vllm_kernel_deltanet_op import device_error, fork_recurrent_state, hybrid_recurrent_forward

__all__ = ["hybrid_recurrent_forward", "fork_recurrent_state", "device_error", "ragged_prefill"]
