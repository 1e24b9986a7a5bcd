"""Serving a compiled model from CUDA graphs: static device batches, pinned
host staging, replay.

The reference serves a model compiled for exactly `batch_size` requests
(`ServingModel`, models/export/compile_entry.py:265-303): every chunk of at
most `batch_size` requests is moved to the device, padded with copies of its
last request, run through the compiled model, and the padding rows are
dropped from the float result; larger batches are split into chunks.

`GraphServingModel.predict` keeps that contract (same argument, same padding
rule, same result, bit for bit: every chunk still runs the same compiled
graph on a full static batch) and changes how a chunk reaches the GPU:

* The compiled forward is captured once per slot into a CUDA graph over
  static device input buffers. A chunk is copied into a slot and the graph
  is replayed: no Python dispatch, no Inductor launcher, no allocation.
* Host inputs cross PCIe on a copy stream, from the caller's pinned tensors
  directly or through pinned staging buffers, so the host-to-device copy of
  chunk i+1 overlaps the forward of chunk i (two slots).
* Padding is done on the device: only the chunk's own rows cross PCIe.

A model compiled with this library's operator (the compile pass rewrites
every RBF-attention site to torch.ops.vectra.rbf_attention) replays its
kernels inside the graph; the operator makes no host synchronisation and no
allocation the capture cannot serve.

A compiled forward that reads a device value on the host cannot be
captured. The reference's price model is one: its radius trim is a
torch.cond (models/price_transformer/model.py:96-138), and Inductor
evaluates the predicate with `.item()` in the generated wrapper before it
picks a branch. `capture=False` serves such a model with everything above
except the graph: the same static slots, device-side padding, pinned
staging and copy/compute overlap, with the compiled forward called on the
slot's static inputs for every chunk.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch


def chunks(n: int, batch_size: int) -> list[tuple[int, int]]:
    """[start, stop) rows of each chunk, in order (the reference's split,
    compile_entry.py:291-293): full chunks of `batch_size`, the last one
    possibly shorter."""
    if batch_size < 1:
        raise ValueError(f'batch_size must be >= 1, got {batch_size}')
    if n < 1:
        raise ValueError(f'a batch needs at least one request, got {n}')
    return [(s, min(s + batch_size, n)) for s in range(0, n, batch_size)]


def pad_in_place(batch: torch.Tensor, size: int) -> torch.Tensor:
    """Rows `size`.. of `batch` become copies of row `size - 1` (the
    reference's padding with the chunk's last request,
    compile_entry.py:296-300); returns `batch`."""
    if not 1 <= size <= batch.shape[0]:
        raise ValueError(f'{size} rows do not fit a batch of '
                         f'{batch.shape[0]}')
    if size < batch.shape[0]:
        batch[size:].copy_(batch[size - 1:size].expand(
            batch.shape[0] - size, *batch.shape[1:]))
    return batch


class _Slot:
    """One static batch: device inputs, the captured graph, its output,
    pinned staging for host inputs, and the events that order reuse."""

    def __init__(self, example: Sequence[torch.Tensor]):
        self.inputs = [torch.empty_like(t) for t in example]
        for dst, src in zip(self.inputs, example):
            dst.copy_(src)
        self.staging = None  # pinned host copies, made on first host chunk
        self.graph = None
        self.output = None
        self.copied = torch.cuda.Event()    # H2D into `inputs` done
        self.released = torch.cuda.Event()  # replay + output copy done
        self.released_valid = False

    def staging_buffers(self):
        if self.staging is None:
            self.staging = [torch.empty(t.shape, dtype=t.dtype,
                                        pin_memory=True)
                            for t in self.inputs]
        return self.staging


class GraphServingModel:
    """A compiled model served by CUDA-graph replay over static batches.

    Args:
      compiled: The compiled forward (e.g. `compile_for_serving`'s result),
        called as compiled(*inputs) on `batch_size`-row device tensors.
      example_inputs: Device tensors of the serving shape; their first
        dimension is the batch size. Their values are used for warm-up and
        capture only.
      slots: Static batches in flight (2: one being copied in while the
        other runs).
      warmup: Eager calls on a side stream before the captures.
      capture: Capture each slot's forward in a CUDA graph (True), or call
        the compiled forward on the slot's inputs for every chunk (False:
        for forwards that synchronise with the host, which a capture
        forbids).

    `predict` is not thread-safe: one instance serves one caller stream.
    """

    def __init__(self, compiled: Callable, example_inputs: Sequence[
            torch.Tensor], slots: int = 2, warmup: int = 2,
                 capture: bool = True):
        example = list(example_inputs)
        if not example:
            raise ValueError('example_inputs is empty')
        device = example[0].device
        if device.type != 'cuda':
            raise ValueError('example_inputs must be CUDA tensors')
        b = example[0].shape[0]
        for t in example:
            if t.device != device or t.dim() < 1 or t.shape[0] != b:
                raise ValueError('example_inputs must share one CUDA device '
                                 'and one batch size (dim 0)')
        if slots < 1:
            raise ValueError(f'slots must be >= 1, got {slots}')
        self.compiled = compiled
        self.captured = bool(capture)
        self.batch_size = b
        self.device = device
        self._shapes = [(t.dtype, tuple(t.shape[1:])) for t in example]
        with torch.cuda.device(device):
            self._copy_stream = torch.cuda.Stream()
            self._slots = [_Slot(example) for _ in range(slots)]
            self._capture(warmup)

    def _capture(self, warmup):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.no_grad(), torch.cuda.stream(side):
            for _ in range(warmup):
                self.compiled(*self._slots[0].inputs)
        torch.cuda.current_stream().wait_stream(side)
        pool = torch.cuda.graph_pool_handle() if self.captured else None
        for slot in self._slots:
            if self.captured:
                slot.graph = torch.cuda.CUDAGraph()
                with torch.no_grad(), torch.cuda.graph(slot.graph, pool=pool):
                    slot.output = self.compiled(*slot.inputs)
            else:
                with torch.no_grad():
                    slot.output = self.compiled(*slot.inputs)
            if not isinstance(slot.output, torch.Tensor):
                raise TypeError('the compiled model must return one tensor')
            if slot.output.dim() < 1 or slot.output.shape[0] != \
                    self.batch_size:
                raise ValueError('the compiled model must return one row '
                                 'per request (dim 0 = batch size)')
        torch.cuda.current_stream().synchronize()

    def _check(self, tensors):
        if len(tensors) != len(self._shapes):
            raise ValueError(f'expected {len(self._shapes)} input tensors, '
                             f'got {len(tensors)}')
        n = tensors[0].shape[0] if tensors[0].dim() else 0
        for t, (dtype, tail) in zip(tensors, self._shapes):
            if t.dim() < 1 or t.shape[0] != n or tuple(t.shape[1:]) != tail:
                raise ValueError(f'input of shape {tuple(t.shape)} does not '
                                 f'match the served shape [n, *{tail}]')
            if t.dtype != dtype:
                raise ValueError(f'input dtype {t.dtype} != served {dtype}')
            if t.device.type not in ('cpu', 'cuda') or (
                    t.device.type == 'cuda' and t.device != self.device):
                raise ValueError(f'input on {t.device}; the model is served '
                                 f'on {self.device}')
        return n

    def predict(self, inputs: Sequence[torch.Tensor]) -> torch.Tensor:
        """The model's output for every request, as float32 on the serving
        device: [n, *output.shape[1:]] for a batch of any size n >= 1.

        Inputs may be host tensors (pinned ones are copied directly,
        others through pinned staging) or tensors on the serving device.
        The result is ordered on the caller's current stream.
        """
        tensors = list(inputs)
        n = self._check(tensors)
        b = self.batch_size
        with torch.cuda.device(self.device):
            compute = torch.cuda.current_stream()
            head = self._slots[0].output
            out = torch.empty((n, *head.shape[1:]), dtype=torch.float32,
                              device=self.device)
            # Inputs produced on the caller's stream are ready for the copy
            # stream too.
            self._copy_stream.wait_stream(compute)
            for i, (start, stop) in enumerate(chunks(n, b)):
                slot = self._slots[i % len(self._slots)]
                size = stop - start
                self._fill(slot, [t[start:stop] for t in tensors], compute)
                compute.wait_event(slot.copied)
                for t in slot.inputs:
                    pad_in_place(t, size)
                if self.captured:
                    slot.graph.replay()
                else:
                    with torch.no_grad():
                        slot.output = self.compiled(*slot.inputs)
                out[start:stop].copy_(slot.output[:size])
                slot.released.record(compute)
                slot.released_valid = True
        return out

    def _fill(self, slot, parts, compute):
        """Copies one chunk's rows into `slot.inputs[:size]` and records
        `slot.copied` (host rows on the copy stream, device rows on the
        caller's stream)."""
        size = parts[0].shape[0]
        on_host = [p.device.type == 'cpu' for p in parts]
        if any(on_host):
            stream = self._copy_stream
            if slot.released_valid:
                # The slot's previous replay must have read its inputs.
                stream.wait_event(slot.released)
            staging = None
            for p, host in zip(parts, on_host):
                if host and not (p.is_pinned() and p.is_contiguous()):
                    # The staging buffers are reused: the previous copy out
                    # of them must have finished.
                    slot.copied.synchronize()
                    staging = slot.staging_buffers()
                    break
            with torch.cuda.stream(stream):
                for j, (dst, p, host) in enumerate(zip(slot.inputs, parts,
                                                       on_host)):
                    if not host:
                        dst[:size].copy_(p, non_blocking=True)
                    elif p.is_pinned() and p.is_contiguous():
                        dst[:size].copy_(p, non_blocking=True)
                    else:
                        staging[j][:size].copy_(p)
                        dst[:size].copy_(staging[j][:size],
                                         non_blocking=True)
            slot.copied.record(stream)
        else:
            for dst, p in zip(slot.inputs, parts):
                dst[:size].copy_(p)
            slot.copied.record(compute)
