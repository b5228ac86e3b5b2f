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
GPU time of a whole forward once it is split 4 or 8 ways.  So host (numpy) batches run as
captured CUDA graphs (NCCL collectives included); the device schedule of each batch
(sequence starts, attention work list) is computed inside the graph from the new
positions, so one graph serves every batch of its token layout.

The engine's batcher packs whole requests up to a token budget
(``core/tokenizer_manager.py:98-139``), so the token count T varies from batch to batch.
A graph is therefore keyed on a *bucketed* layout: the batch (each tensor-parallel
micro-batch separately) is padded up to the next bucket size (multiples of 256 tokens up
to 32768, of 2048 up to 131072, of 8192 beyond: about 1% padding at 20 k tokens) with dummy
sequences of at most 128 tokens, whose rows are never pooled and cost almost no attention.
A new T then reuses the graph of its bucket, and a stream of varying batches settles on a
fixed set of graphs.  A layout that keeps repeating exactly (``exact_after`` times) gets a
graph of its own, without padding.  A capture costs about three forwards, so this pays
only for shapes that recur many times.  Every row of a real token is computed exactly as
in the unpadded forward (row results of every kernel are independent of the other rows of
batches of more than 256 tokens, and the dummy sequences attend only to themselves).  All
graphs share one memory pool, so holding several costs the memory of the largest, not
their sum.

Last rows only (``last_rows_only=True`` or ``MES_LAST_ROWS_ONLY=1``; off by default).  The
post-process pools one token per sequence, so ``embed`` can run the last layer's o_proj, MLP
and final norm on those B rows alone (``DecoderModel.forward_last_rows``); the embeddings
are the same, and ``_inference`` (all rows) is unaffected.  The graph of such a batch also
holds the row indices (padded to a multiple of 16 with row 0; the extra rows are dropped).
"""
from __future__ import annotations

import collections
import os
import warnings

import numpy as np
import torch
import torch.distributed as dist

from ..models.qwen2 import DecoderModel
from ..models.registry import get_model_class
from ..ultils.pool import last_token_l2

PAD_SEQ = 128   # longest dummy sequence used for padding


def tp_nccl_environment(world_size: int | None = None) -> None:
    """Call before ``init_process_group`` at tensor parallelism > 1 (``world_size``
    defaults to ``WORLD_SIZE``).  The model overlaps each all-reduce with the other
    micro-batch's kernels and keeps ``DecoderModel.overlap_reserved_sms(world_size)`` SMs
    free for it; capping NCCL's ring/tree channels (one CTA each) at as many keeps the
    collective inside them.  Settings already in the environment win."""
    world = int(world_size if world_size is not None else os.environ.get("WORLD_SIZE", "1"))
    os.environ.setdefault("NCCL_MAX_NCHANNELS", str(max(DecoderModel.overlap_reserved_sms(world), 1)))


def token_bucket(n: int) -> int:
    """Padded token count of a (micro-)batch of ``n`` tokens: the next multiple of 256 up
    to 32768, of 2048 up to 131072, of 8192 beyond (at most 256 / n, 2048 / n or
    8192 / n padding: ~1.3% at 20 k tokens)."""
    step = 256 if n <= 32768 else 2048 if n <= 131072 else 8192
    return max(step, -(-n // step) * step)


class Layout:
    """Where the tokens of a host batch go in the (padded) device batch.

    ``parts``: ``(src_start, src_end, dst_start, padded_len)`` per micro-batch (one part
    unsplit, two at tp > 1 when the batch is split at a sequence boundary); ``split``: the
    device micro-batch boundary handed to the model (``DecoderModel.NO_SPLIT`` when
    unsplit)."""

    def __init__(self, parts, split: int):
        self.parts = tuple(parts)
        self.split = split
        self.total = sum(p[3] for p in self.parts)
        self.padded = any(p[1] - p[0] != p[3] for p in self.parts)

    @property
    def key(self):
        return (tuple(p[3] for p in self.parts), self.split)

    def pad(self, ids: np.ndarray, pos: np.ndarray):
        """Padded copies of ``ids`` / ``positions`` (dummy sequences of <= PAD_SEQ tokens,
        id 0, positions restarting at 0 so that each starts a new sequence)."""
        if not self.padded:
            return ids, pos
        out_ids = np.zeros(self.total, dtype=np.int64)
        out_pos = np.empty(self.total, dtype=np.int64)
        for s0, s1, d0, n in self.parts:
            m = s1 - s0
            out_ids[d0:d0 + m] = ids[s0:s1]
            out_pos[d0:d0 + m] = pos[s0:s1]
            out_pos[d0 + m:d0 + n] = np.arange(n - m) % PAD_SEQ
        return out_ids, out_pos

    def rows(self, idx):
        """Device rows of host token indices ``idx``: a numpy array for a list or array, an
        int64 tensor on the same device for a tensor (mapped there, without a host
        synchronisation)."""
        if isinstance(idx, torch.Tensor):
            idx = idx.to(torch.int64)
            out = idx.clone()
            for s0, s1, d0, _ in self.parts:
                out = torch.where((idx >= s0) & (idx < s1), idx - s0 + d0, out)
            return out
        idx = np.asarray(idx, dtype=np.int64)
        out = idx.copy()
        for s0, s1, d0, _ in self.parts:
            sel = (idx >= s0) & (idx < s1)
            out[sel] = idx[sel] - s0 + d0
        return out


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
        self.tp_size = getattr(self.model, "tp_size", self.world_size)
        self.last_rows_only = os.environ.get("MES_LAST_ROWS_ONLY", "0") == "1"
        self.use_cuda_graphs = os.environ.get("MES_CUDA_GRAPHS", "1") != "0"
        self.max_graphs = 128        # bucketed layouts kept (least recently used dropped)
        self.max_exact_graphs = 8    # exact layouts of repeated token counts kept
        self.exact_after = 8         # occurrences of an exact layout before it gets a graph
        self._graphs: collections.OrderedDict = collections.OrderedDict()
        self._exact: collections.OrderedDict = collections.OrderedDict()
        self._seen: collections.Counter = collections.Counter()
        self._no_graph: set = set()
        self._pool = None
        self.captures = 0            # graphs captured so far (for tests and benchmarks)
        self._staging: dict = {}     # name -> (pinned host buffer, event of its last copy)

    def _to_device(self, array) -> torch.Tensor:
        t = torch.from_numpy(np.ascontiguousarray(array)) if isinstance(array, np.ndarray) else array
        if t.device.type == "cpu":
            t = t.pin_memory().to(self.device, non_blocking=True)
        return t

    def _upload(self, name: str, array, dst: torch.Tensor | None = None) -> torch.Tensor:
        """Asynchronous host-to-device copy of the int64 host ``array`` into ``dst`` (a new
        device tensor if None) through a pinned staging buffer kept per ``name``; the buffer
        is reused once its previous copy has completed."""
        a = np.asarray(array, dtype=np.int64).reshape(-1)
        n = a.shape[0]
        buf, ev = self._staging.get(name, (None, None))
        if buf is None or buf.shape[0] < n:
            buf = torch.empty(max(n, 4096), dtype=torch.int64, pin_memory=True)
            ev = torch.cuda.Event()
        else:
            ev.synchronize()
        buf.numpy()[:n] = a
        if dst is None:
            dst = torch.empty(n, dtype=torch.int64, device=self.device)
        dst.copy_(buf[:n], non_blocking=True)
        ev.record(torch.cuda.current_stream(self.device))
        self._staging[name] = (buf, ev)
        return dst

    # ---------------------------------------------------------------- layouts and graphs
    def layout(self, positions, exact: bool = False, split: int | None = None) -> Layout:
        """Device layout of a host batch: its micro-batch boundary (tp > 1; ``split`` when
        the caller already has it from :meth:`DecoderModel.overlap_split_host`) and, unless
        ``exact``, each micro-batch padded to its token bucket."""
        pos = np.asarray(positions)
        T = int(pos.shape[0])
        if split is None:
            split = DecoderModel.overlap_split_host(pos, self.tp_size)
        if split == DecoderModel.NO_SPLIT:
            spans = [(0, T)]
        else:
            spans = [(0, split), (split, T)]
        parts, d0 = [], 0
        for s0, s1 in spans:
            n = s1 - s0 if exact else token_bucket(s1 - s0)
            parts.append((s0, s1, d0, n))
            d0 += n
        dev_split = DecoderModel.NO_SPLIT if len(parts) == 1 else parts[1][2]
        return Layout(parts, dev_split)

    def _graph_layout(self, positions) -> Layout:
        """Layout to run a host batch with: exact when its graph exists, its layout needs no
        padding, or it has now occurred ``exact_after`` times; else bucketed."""
        split = DecoderModel.overlap_split_host(np.asarray(positions), self.tp_size)
        exact = self.layout(positions, exact=True, split=split)
        if any(k[0] == exact.key for k in self._exact):
            return exact
        bucket = self.layout(positions, split=split)
        if not bucket.padded:
            return exact
        if len(self._seen) > 4096:       # forget old shapes; the counts only pick exact graphs
            self._seen.clear()
        self._seen[exact.key] += 1
        return exact if self._seen[exact.key] >= self.exact_after else bucket

    def _graph_for(self, lay: Layout, ids, pos, n_rows: int = 0):
        """The captured forward of layout ``lay`` (with ``n_rows`` last rows, see
        :meth:`capture`), captured on first use; None if capture failed (that layout then
        runs eagerly)."""
        cache, limit = (self._graphs, self.max_graphs) if lay.padded else (self._exact, self.max_exact_graphs)
        key = (lay.key, n_rows)
        g = cache.get(key)
        if g is not None:
            cache.move_to_end(key)
            return g
        try:
            g = self.capture(lay, ids, pos, n_rows)
        except Exception as exc:   # an unsupported capture runs eagerly from now on
            warnings.warn(f"CUDA-graph capture of a {lay.total}-token batch failed ({exc!r}); "
                          "batches of this layout run eagerly", RuntimeWarning, stacklevel=2)
            self._no_graph.add(key)
            return None
        cache[key] = g
        while len(cache) > limit:
            cache.popitem(last=False)
        return g

    @torch.no_grad()
    def capture(self, lay: Layout, input_ids, positions, n_rows: int = 0):
        """Capture one forward of layout ``lay`` into a CUDA graph (memory from the worker's
        shared graph pool).  Returns ``(graph, ids, positions, rows, out)``: the static
        device input buffers to fill (padded) before ``graph.replay()`` and the output it
        writes - ``[lay.total, H]``, or with ``n_rows`` > 0 the final states ``[n_rows, H]``
        of the rows listed in ``rows`` (int64 [n_rows]; :meth:`DecoderModel.forward_last_rows`).
        ``input_ids`` / ``positions``: a host batch of that layout (not yet padded), run
        once eagerly first."""
        ids_h, pos_h = lay.pad(np.asarray(input_ids), np.asarray(positions))
        ids_s = torch.empty(lay.total, dtype=torch.int64, device=self.device)
        pos_s = torch.empty(lay.total, dtype=torch.int64, device=self.device)
        rows_s = torch.zeros(n_rows, dtype=torch.int64, device=self.device) if n_rows else None
        ids_s.copy_(self._to_device(ids_h))
        pos_s.copy_(self._to_device(pos_h))

        def run():
            if n_rows:
                return self.model.forward_last_rows(ids_s, pos_s, rows_s)
            return self.model(ids_s, pos_s, overlap_split=lay.split)

        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            run()
        torch.cuda.current_stream(self.device).wait_stream(side)
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._pool):
            out = run()
        self.captures += 1
        return graph, ids_s, pos_s, rows_s, out

    def release_graphs(self) -> None:
        """Drop every captured graph (required before the process group is destroyed when
        the graphs hold NCCL work)."""
        self._graphs.clear()
        self._exact.clear()

    # ---------------------------------------------------------------- forward
    def _hidden_size(self) -> int:
        cfg = getattr(self.mes_config, "model_config", None)
        if cfg is not None:
            return int(cfg.hidden_size)
        return int(self.model.model.embed_tokens.embedding_dim)

    @torch.no_grad()
    def _forward(self, input_ids, positions, last_token_indices=None):
        """Forward of one batch: ``(hidden, layout)``.  ``hidden`` holds the model output in
        the device layout (``layout.rows`` maps host token indices to its rows; ``layout``
        is None for an unpadded eager forward) - or, when ``last_token_indices`` is given
        and the last-rows forward applies, the final states of exactly those tokens, in
        their order (``layout`` is then the string "rows")."""
        host = not (isinstance(positions, torch.Tensor) and positions.is_cuda)
        rows_mode = last_token_indices is not None
        if self.use_cuda_graphs and host:
            ids_h = np.asarray(input_ids.numpy() if isinstance(input_ids, torch.Tensor) else input_ids)
            pos_h = np.asarray(positions.numpy() if isinstance(positions, torch.Tensor) else positions)
            lay = self._graph_layout(pos_h)
            # The last-rows graph takes host row indices (device ones pool the full output).
            rows_mode = (rows_mode and lay.split == DecoderModel.NO_SPLIT
                         and not (isinstance(last_token_indices, torch.Tensor)
                                  and last_token_indices.is_cuda))
            n_rows = -(-len(last_token_indices) // 16) * 16 if rows_mode else 0
            if (lay.key, n_rows) not in self._no_graph:
                g = self._graph_for(lay, ids_h, pos_h, n_rows)
                if g is not None:
                    graph, ids_s, pos_s, rows_s, out = g
                    ids_p, pos_p = lay.pad(ids_h, pos_h)
                    self._upload("ids", ids_p, ids_s)
                    self._upload("positions", pos_p, pos_s)
                    if rows_mode:
                        rows = np.zeros(n_rows, dtype=np.int64)
                        rows[:len(last_token_indices)] = lay.rows(last_token_indices)
                        self._upload("rows", rows, rows_s)
                    graph.replay()
                    if rows_mode:
                        return out[:len(last_token_indices)], "rows"
                    return out, lay
        input_ids = self._to_device(input_ids).to(torch.int64)
        positions = self._to_device(positions).to(torch.int64)
        if rows_mode and (self.tp_size == 1 or self.model.model._overlap_split(positions) is None):
            rows = self._to_device(torch.as_tensor(last_token_indices, dtype=torch.int64))
            return self.model.forward_last_rows(input_ids, positions, rows), "rows"
        return self.model(input_ids=input_ids, positions=positions), None

    @torch.no_grad()
    def _inference(self, input_ids, positions) -> torch.Tensor:
        """``[T, H]`` hidden states of the batch (``gpu_worker.py:216-222``).  With CUDA
        graphs the result lives in the graph's output buffer: it is overwritten by the
        next call."""
        if len(positions) == 0:
            return torch.empty(0, self._hidden_size(), dtype=torch.bfloat16, device=self.device)
        out, lay = self._forward(input_ids, positions)
        if lay is None or not lay.padded:
            return out
        if len(lay.parts) == 1:
            return out[: lay.parts[0][1]]
        return torch.cat([out[d0:d0 + (s1 - s0)] for s0, s1, d0, _ in lay.parts])

    @torch.no_grad()
    def postprocess(self, outputs: torch.Tensor, last_token_indices) -> torch.Tensor:
        """fp32 ``[B, H]`` host tensor of L2-normalised last-token states."""
        idx = last_token_indices
        if not (isinstance(idx, torch.Tensor) and idx.is_cuda):
            idx = self._upload("last", idx.numpy() if isinstance(idx, torch.Tensor) else idx)
        emb = last_token_l2(outputs, idx)
        # One pinned result buffer, reused: the caller gets a copy of it.
        out = getattr(self, "_host_out", None)
        if out is None or out.numel() < emb.numel():
            out = self._host_out = torch.empty(max(emb.numel(), 1 << 16), dtype=torch.float32,
                                               pin_memory=True)
        host = out[:emb.numel()].view(emb.shape)
        host.copy_(emb, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return host.clone()

    def embed(self, input_ids, positions, last_token_indices) -> torch.Tensor:
        """fp32 ``[B, H]`` embeddings: ``_inference`` + ``postprocess`` (the engine's call
        per batch).  A batch without sequences gives ``[0, H]`` and launches nothing."""
        if len(last_token_indices) == 0:
            return torch.empty(0, self._hidden_size(), dtype=torch.float32)
        if self.last_rows_only:
            out, lay = self._forward(input_ids, positions, last_token_indices)
            if lay == "rows":
                return self.postprocess(out, np.arange(out.shape[0]))
        else:
            out, lay = self._forward(input_ids, positions)
        if lay is not None and lay.padded:
            last_token_indices = lay.rows(last_token_indices)
        return self.postprocess(out, last_token_indices)

    def embed_list(self, input_ids, positions, last_token_indices) -> list[list[float]]:
        """The reference's wire format: one Python list of floats per sequence
        (``gpu_worker.py:264-267``)."""
        return self.embed(input_ids, positions, last_token_indices).tolist()
