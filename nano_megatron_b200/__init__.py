"""nano_megatron_b200: a Blackwell-native (sm_100a) mini-Megatron GPT training framework."""

__version__ = "0.1.0"
