"""``last_token_pool`` (``ultils/pool.py:4-9``)."""
import torch


def last_token_pool(hidden_states: torch.Tensor, seq_len: int) -> torch.Tensor:
    return hidden_states[seq_len - 1]
