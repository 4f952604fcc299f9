"""Continuous batching and prefill chunking feeding the grouped INT4 MoE kernel.

The request bookkeeping keeps the interface and behaviour of HydraNet's
scheduler (``scheduler/continuous_batch.py``): ``Request`` / ``RequestState``
/ ``Batch`` (``:21-85``), ``ContinuousBatcher`` (``:88-208``: a bounded
pending queue, batches that keep the active requests first and admit
pending ones up to ``max_batch_size``), ``MicrobatchScheduler`` (``:211-262``:
prompt split into micro-batches, "same experts next" prefetch guess) and
``PrefetchSchedule`` (``:383-439``).  In the reference nothing calls them.

``MoEBatchRunner`` is what wires them to the hot path: every step takes the
batcher's current batch, gives each prefilling request its next chunk of
prompt positions (at most ``prefill_chunk``) and each generating request one
position, concatenates them into ONE token matrix -- prefill chunks and
decode tokens of different requests side by side -- copies it to the device
in one pinned host-to-device copy, runs every MoE layer ONCE over the whole
matrix (the grouped kernel plans per expert across all requests, so an
expert's weights are read once per step however many requests touch it), and
reads the result back in one copy, split per request.  Routing is per token,
so a token's output does not depend on which requests share its step.

The path carries hidden states, not token ids: embedding, attention and the
sampler are outside the MoE hot path.  A request's prompt is its
``prompt_hidden`` rows; after the prompt, each generated position's input is
produced by ``next_input`` from the previous position's output (by default the
output rescaled to the RMS of a unit-variance row), a stand-in for the rest of
the model.
"""

from __future__ import annotations

import threading
import time
from collections import deque
from dataclasses import dataclass, field
from enum import Enum
from typing import Callable, Dict, List, Optional, Sequence, Set, Tuple

import torch


class RequestState(Enum):
    """``scheduler/continuous_batch.py:21-27``."""
    PENDING = "pending"
    PREFILLING = "prefilling"
    GENERATING = "generating"
    COMPLETED = "completed"
    CANCELLED = "cancelled"


@dataclass
class Request:
    """One generation request (``scheduler/continuous_batch.py:30-58``), plus the
    MoE path's inputs: ``prompt_hidden`` [prompt_len, H] and how many prompt
    positions have been run (``prefill_pos``); ``outputs`` collects the layer
    stack's output row of every position run, in position order."""
    request_id: str
    prompt_ids: torch.Tensor
    max_tokens: int = 256
    temperature: float = 0.8
    top_k: int = 50
    top_p: float = 0.9
    state: RequestState = RequestState.PENDING
    generated_ids: List[int] = field(default_factory=list)
    kv_cache_position: int = 0
    submit_time: float = field(default_factory=time.time)
    start_time: Optional[float] = None
    end_time: Optional[float] = None
    prompt_hidden: Optional[torch.Tensor] = None
    prefill_pos: int = 0
    inputs: List[torch.Tensor] = field(default_factory=list)
    outputs: List[torch.Tensor] = field(default_factory=list)

    @property
    def total_tokens(self) -> int:
        return len(self.prompt_ids) + len(self.generated_ids)

    @property
    def is_active(self) -> bool:
        return self.state in (RequestState.PREFILLING, RequestState.GENERATING)


@dataclass
class Batch:
    """Requests processed together in one step (``scheduler/continuous_batch.py:61-85``)."""
    requests: List[Request]
    batch_id: int
    input_ids: Optional[torch.Tensor] = None
    position_ids: Optional[torch.Tensor] = None
    kv_indices: Optional[List[int]] = None

    @property
    def batch_size(self) -> int:
        return len(self.requests)

    @property
    def is_prefill(self) -> bool:
        return any(r.state == RequestState.PREFILLING for r in self.requests)


class ContinuousBatcher:
    """Request queue that forms a batch every step (``scheduler/continuous_batch.py:88-208``).

    A batch holds the active requests (in admission order) and then pending
    ones, oldest first, up to ``max_batch_size``; an admitted request becomes
    PREFILLING.  ``submit`` refuses requests while ``max_queue_size`` are
    pending.  Thread-safe: ``get_batch`` waits up to its timeout for work."""

    def __init__(self, max_batch_size: int = 8, max_queue_size: int = 64, batch_timeout_ms: float = 10.0):
        self.max_batch_size = max_batch_size
        self.max_queue_size = max_queue_size
        self.batch_timeout_ms = batch_timeout_ms
        self.pending_queue: deque = deque()
        self.active_requests: Dict[str, Request] = {}
        self.completed_requests: Dict[str, Request] = {}
        self.next_batch_id = 0
        self._lock = threading.Lock()
        self._queue_not_empty = threading.Condition(self._lock)

    def submit(self, request: Request) -> bool:
        with self._lock:
            if len(self.pending_queue) >= self.max_queue_size:
                return False
            request.state = RequestState.PENDING
            self.pending_queue.append(request)
            self._queue_not_empty.notify()
            return True

    def get_batch(self, timeout_ms: Optional[float] = None) -> Optional[Batch]:
        deadline = time.time() + (timeout_ms or self.batch_timeout_ms) / 1000.0
        with self._lock:
            while True:
                batch = self._try_form_batch()
                if batch is not None:
                    return batch
                left = deadline - time.time()
                if left <= 0:
                    return None
                self._queue_not_empty.wait(timeout=left)

    def _try_form_batch(self) -> Optional[Batch]:
        chosen = [r for r in self.active_requests.values() if r.is_active][:self.max_batch_size]
        while self.pending_queue and len(chosen) < self.max_batch_size:
            r = self.pending_queue.popleft()
            r.state = RequestState.PREFILLING
            r.start_time = time.time()
            self.active_requests[r.request_id] = r
            chosen.append(r)
        if not chosen:
            return None
        batch = Batch(requests=chosen, batch_id=self.next_batch_id)
        self.next_batch_id += 1
        return batch

    def _finish(self, request_id: str, state: RequestState, stamp: bool):
        with self._lock:
            r = self.active_requests.pop(request_id, None)
            if r is None:
                return
            r.state = state
            if stamp:
                r.end_time = time.time()
            self.completed_requests[request_id] = r

    def complete_request(self, request_id: str):
        self._finish(request_id, RequestState.COMPLETED, True)

    def cancel_request(self, request_id: str):
        self._finish(request_id, RequestState.CANCELLED, False)

    def get_stats(self) -> Dict:
        with self._lock:
            return {"pending_count": len(self.pending_queue), "active_count": len(self.active_requests),
                    "completed_count": len(self.completed_requests)}


class MicrobatchScheduler:
    """Prompt split into micro-batches of ``microbatch_size`` positions
    (``scheduler/continuous_batch.py:211-262``)."""

    def __init__(self, microbatch_size: int = 4, num_prefetch_streams: int = 2):
        self.microbatch_size = microbatch_size
        self.num_prefetch_streams = num_prefetch_streams

    def split_prefill(self, input_ids: torch.Tensor) -> List[Tuple[torch.Tensor, int]]:
        """[(input_ids[:, s:s+m], s)] over the sequence dimension."""
        n = input_ids.shape[1]
        return [(input_ids[:, s:min(s + self.microbatch_size, n)], s) for s in range(0, n, self.microbatch_size)]

    def get_prefetch_experts(self, current_mb_experts: List[Tuple[int, int]], next_mb_idx: int,
                             total_mbs: int) -> List[Tuple[int, int]]:
        """The next micro-batch is guessed to use the current one's experts."""
        return [] if next_mb_idx >= total_mbs else current_mb_experts


class PrefetchSchedule:
    """(layer, expert, stream) prefetches for the next micro-batch, each
    (layer, expert) once until ``clear`` (``scheduler/continuous_batch.py:383-439``)."""

    def __init__(self, num_layers: int, num_experts: int, num_streams: int = 2):
        self.num_layers = num_layers
        self.num_experts = num_experts
        self.num_streams = num_streams
        self.prefetched: Set[Tuple[int, int]] = set()
        self.stream_idx = 0

    def schedule_prefetch(self, current_layer: int, current_experts: List[int],
                          next_mb_experts: Optional[List[int]] = None) -> List[Tuple[int, int, int]]:
        out = []
        for e in next_mb_experts or []:
            key = (current_layer, e)
            if key in self.prefetched:
                continue
            out.append((current_layer, e, self.stream_idx % self.num_streams))
            self.stream_idx += 1
            self.prefetched.add(key)
        return out

    def clear(self):
        self.prefetched.clear()
        self.stream_idx = 0


def rms_feedback(prev_out: torch.Tensor) -> torch.Tensor:
    """Default ``next_input``: the previous position's output rescaled to unit RMS."""
    x = prev_out.float()
    return (x * torch.rsqrt(x.pow(2).mean().clamp_min(1e-12))).to(prev_out.dtype)


@dataclass
class StepRecord:
    """What one runner step did: batch id, (request id, first position, rows) per
    request in matrix order, and the number of rows."""
    batch_id: int
    parts: List[Tuple[str, int, int]]
    rows: int
    prefill_rows: int
    decode_rows: int


class MoEBatchRunner:
    """Runs a stack of token-wise layers (``MoELayerInt4``, ``SlotCachedMoELayer``,
    ``ExpertParallelMoE`` ...: modules mapping [n, H] -> [n, H]) over the
    batcher's requests, one grouped call per layer per step.

    A request is complete once its prompt has run and ``max_tokens`` positions
    have been generated after it (the last prompt position's output feeds the
    first generated position).  ``step`` returns None when there was nothing
    to run."""

    def __init__(self, layers: Sequence[torch.nn.Module], batcher: ContinuousBatcher, hidden_dim: int,
                 prefill_chunk: int = 256, device: Optional[torch.device] = None, dtype=torch.bfloat16,
                 next_input: Callable[[torch.Tensor], torch.Tensor] = rms_feedback, keep_inputs: bool = False):
        if prefill_chunk < 1:
            raise ValueError("prefill_chunk must be at least 1")
        self.layers = list(layers)
        self.batcher = batcher
        self.H = hidden_dim
        self.prefill_chunk = prefill_chunk
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.dtype = dtype
        self.next_input = next_input
        self.keep_inputs = keep_inputs
        self.records: List[StepRecord] = []
        pin = self.device.type == "cuda"
        self._pin = pin
        self._host_in = torch.empty(0, hidden_dim, dtype=dtype)
        self._host_out = torch.empty(0, hidden_dim, dtype=dtype)

    def _buffers(self, n: int):
        if self._host_in.shape[0] < n:
            cap = max(n, 2 * self._host_in.shape[0])
            self._host_in = torch.empty(cap, self.H, dtype=self.dtype, pin_memory=self._pin)
            self._host_out = torch.empty(cap, self.H, dtype=self.dtype, pin_memory=self._pin)
        return self._host_in[:n], self._host_out[:n]

    def _rows_of(self, r: Request) -> torch.Tensor:
        """Host rows this request contributes to the step (not yet consumed)."""
        if r.state == RequestState.PREFILLING:
            if r.prompt_hidden is None or r.prompt_hidden.shape[0] == 0:
                raise ValueError(f"request {r.request_id} has no prompt rows")
            return r.prompt_hidden[r.prefill_pos:r.prefill_pos + self.prefill_chunk]
        return self.next_input(r.outputs[-1]).view(1, self.H)

    def step(self) -> Optional[StepRecord]:
        batch = self.batcher.get_batch(timeout_ms=0.001)  # no waiting: the runner drives the steps
        if batch is None:
            return None
        pieces = [(r, self._rows_of(r)) for r in batch.requests]
        n = sum(p.shape[0] for _, p in pieces)
        host_in, host_out = self._buffers(n)
        parts, o, n_pre = [], 0, 0
        for r, rows in pieces:
            m = rows.shape[0]
            host_in[o:o + m].copy_(rows)
            first = r.prefill_pos if r.state == RequestState.PREFILLING else len(r.prompt_hidden) + len(r.generated_ids)
            parts.append((r.request_id, first, m))
            if r.state == RequestState.PREFILLING:
                n_pre += m
            o += m
        x = host_in.to(self.device, non_blocking=True)
        with torch.no_grad():
            for layer in self.layers:
                x = layer(x)
        host_out.copy_(x, non_blocking=self._pin)
        if self._pin:
            torch.cuda.current_stream(self.device).synchronize()
        o = 0
        for r, rows in pieces:
            m = rows.shape[0]
            out = host_out[o:o + m].clone()
            if self.keep_inputs:
                r.inputs.extend(rows.clone().unbind(0))
            r.outputs.extend(out.unbind(0))
            if r.state == RequestState.PREFILLING:
                r.prefill_pos += m
                r.kv_cache_position = r.prefill_pos
                if r.prefill_pos >= r.prompt_hidden.shape[0]:
                    r.state = RequestState.GENERATING
            else:
                r.generated_ids.append(len(r.generated_ids))
                r.kv_cache_position += 1
            o += m
            if r.state == RequestState.GENERATING and len(r.generated_ids) >= r.max_tokens:
                self.batcher.complete_request(r.request_id)
        rec = StepRecord(batch.batch_id, parts, n, n_pre, n - n_pre)
        self.records.append(rec)
        return rec

    def run(self, max_steps: int = 1_000_000) -> int:
        """Steps until no request is pending or active; returns the steps taken."""
        steps = 0
        while steps < max_steps and self.step() is not None:
            steps += 1
        return steps
