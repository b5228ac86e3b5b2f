"""The hot path of the reference's ``GPUWorker`` (``core/gpu_worker.py``).

``_inference`` copies the packed ``input_ids`` / ``positions`` batch to the device and runs
the model (``gpu_worker.py:216-222``); ``postprocess`` gathers each sequence's last token
and L2-normalises it (``:252-267``) in one fused kernel, producing fp32 on the device and
copying it to the host once.  ``embed`` is the two together - the call the engine's
inference thread makes per batch.  The process shell around it (queues, shared-memory
control plane, callback threads) belongs to the server and is not part of this package.

Every rank of a tensor-parallel group runs ``_inference`` on the same batch; only rank 0
post-processes, as in the reference.

CUDA graphs.  A forward launches about 230 kernels (twice that with the tensor-parallel
micro-batch overlap), and issuing them from Python costs about 60 us each - as much as the
GPU time of a whole forward once it is split 4 or 8 ways.  So ``_inference`` captures the
forward of each batch shape it meets - the token count and, at tp > 1, the micro-batch
boundary - into a CUDA graph (NCCL collectives included) and replays it for later batches
of that shape; the device schedule of each batch (sequence starts, attention work list)
is computed inside the graph from the new positions.  Host (numpy) inputs take this path;
device tensors, whose boundaries would need a host read, run eagerly.
"""
from __future__ import annotations

import collections
import os
import warnings

import numpy as np
import torch
import torch.distributed as dist

from .. import _C
from ..models.qwen2 import DecoderModel
from ..models.registry import get_model_class


def tp_nccl_environment(world_size: int | None = None) -> None:
    """Call before ``init_process_group`` at tensor parallelism > 1 (``world_size``
    defaults to ``WORLD_SIZE``).  The model overlaps each all-reduce with the other
    micro-batch's kernels and keeps ``DecoderModel.overlap_reserved_sms(world_size)`` SMs
    free for it; capping NCCL's ring/tree channels (one CTA each) at as many keeps the
    collective inside them.  Settings already in the environment win."""
    world = int(world_size if world_size is not None else os.environ.get("WORLD_SIZE", "1"))
    os.environ.setdefault("NCCL_MAX_NCHANNELS", str(max(DecoderModel.overlap_reserved_sms(world), 1)))


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
        self.use_cuda_graphs = os.environ.get("MES_CUDA_GRAPHS", "1") != "0"
        self.max_graphs = 8
        self._graphs: collections.OrderedDict = collections.OrderedDict()
        self._no_graph: set = set()

    def _to_device(self, array) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(array)) if isinstance(array, np.ndarray) else array
        if t.device.type == "cpu":
            t = t.pin_memory().to(self.device, non_blocking=True)
        return t

    @torch.no_grad()
    def _inference(self, input_ids, positions) -> torch.Tensor:
        host = not (isinstance(positions, torch.Tensor) and positions.is_cuda)
        if self.use_cuda_graphs and host:
            pos_h = np.asarray(positions.numpy() if isinstance(positions, torch.Tensor) else positions)
            split = DecoderModel.overlap_split_host(pos_h)
            key = (int(pos_h.shape[0]), split)
            if key not in self._no_graph:
                g = self._graph_for(key, input_ids, positions)
                if g is not None:
                    graph, ids_s, pos_s, out = g
                    ids_s.copy_(self._to_device(input_ids).to(torch.int64), non_blocking=True)
                    pos_s.copy_(self._to_device(positions).to(torch.int64), non_blocking=True)
                    graph.replay()
                    return out
        input_ids = self._to_device(input_ids).to(torch.int64)
        positions = self._to_device(positions).to(torch.int64)
        return self.model(input_ids=input_ids, positions=positions)

    def _graph_for(self, key, input_ids, positions):
        """The captured forward for batch shape ``key`` (captured on first use, least
        recently used dropped beyond ``max_graphs``); None if capture failed."""
        g = self._graphs.get(key)
        if g is not None:
            self._graphs.move_to_end(key)
            return g
        try:
            g = self.capture(key[0], key[1], input_ids, positions)
        except Exception as exc:   # an unsupported capture runs eagerly from now on
            warnings.warn(f"CUDA-graph capture of a {key[0]}-token batch failed ({exc!r}); "
                          "batches of this shape run eagerly", RuntimeWarning, stacklevel=2)
            self._no_graph.add(key)
            return None
        self._graphs[key] = g
        while len(self._graphs) > self.max_graphs:
            self._graphs.popitem(last=False)
        return g

    @torch.no_grad()
    def capture(self, T: int, split, input_ids, positions):
        """Capture one forward of a ``T``-token batch (micro-batch boundary ``split``) into a
        CUDA graph with its own memory pool.  Returns ``(graph, ids, positions, out)``: the
        static input buffers to fill before ``graph.replay()`` and the output it writes.
        ``input_ids`` / ``positions`` are a batch of that shape, run once eagerly first."""
        ids_s = torch.empty(T, dtype=torch.int64, device=self.device)
        pos_s = torch.empty(T, dtype=torch.int64, device=self.device)
        ids_s.copy_(self._to_device(input_ids).to(torch.int64))
        pos_s.copy_(self._to_device(positions).to(torch.int64))
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self.model(ids_s, pos_s, overlap_split=split)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = self.model(ids_s, pos_s, overlap_split=split)
        return graph, ids_s, pos_s, out

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
