"""The hot path of the reference's ``GPUWorker`` (``core/gpu_worker.py``).

``_inference`` copies the packed ``input_ids`` / ``positions`` batch to the device and runs
the model (``gpu_worker.py:216-222``); ``postprocess`` gathers each sequence's last token
and L2-normalises it (``:252-267``) in one fused kernel, producing fp32 on the device and
copying it to the host once.  ``embed`` is the two together - the call the engine's
inference thread makes per batch.  The process shell around it (queues, shared-memory
control plane, callback threads) belongs to the server and is not part of this package.

Every rank of a tensor-parallel group runs ``_inference`` on the same batch; only rank 0
post-processes, as in the reference.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .. import _C
from ..models.registry import get_model_class


class GPUWorker:

    def __init__(self, mes_config, device: torch.device | str | None = None, model=None):
        self.mes_config = mes_config
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        if dist.is_available() and dist.is_initialized():
            self.rank, self.world_size = dist.get_rank(), dist.get_world_size()
        else:
            self.rank, self.world_size = 0, 1
        if model is None:
            with torch.device(self.device):
                model = get_model_class(mes_config.model_config)(mes_config)
        self.model = model.eval()

    def _to_device(self, array) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(array)) if isinstance(array, np.ndarray) else array
        if t.device.type == "cpu":
            t = t.pin_memory().to(self.device, non_blocking=True)
        return t

    @torch.no_grad()
    def _inference(self, input_ids, positions) -> torch.Tensor:
        input_ids = self._to_device(input_ids).to(torch.int64)
        positions = self._to_device(positions).to(torch.int64)
        return self.model(input_ids=input_ids, positions=positions)

    @torch.no_grad()
    def postprocess(self, outputs: torch.Tensor, last_token_indices) -> torch.Tensor:
        """fp32 ``[B, H]`` host tensor of L2-normalised last-token states."""
        idx = self._to_device(torch.as_tensor(last_token_indices, dtype=torch.int64))
        emb = _C.last_token_l2(outputs, idx)
        host = torch.empty(emb.shape, dtype=torch.float32, pin_memory=True)
        host.copy_(emb, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return host

    def embed(self, input_ids, positions, last_token_indices) -> torch.Tensor:
        return self.postprocess(self._inference(input_ids, positions), last_token_indices)

    def embed_list(self, input_ids, positions, last_token_indices) -> list[list[float]]:
        """The reference's wire format: one Python list of floats per sequence
        (``gpu_worker.py:264-267``)."""
        return self.embed(input_ids, positions, last_token_indices).tolist()
