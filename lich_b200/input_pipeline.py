"""Pinned-host -> device input pipeline for the training loop.

The reference copies every batch synchronously inside ``prepare_batch``
(``src/ipc_tilelang/trainer.py:836-846``) and lists an asynchronous input
pipeline as pending (``README.md:171-172``).  ``BatchPipeline`` keeps a ring
of ``depth`` device slots fed from pinned host memory on a dedicated copy
stream, so the copy of the next batch runs under the training step of the
current one.  ``source`` yields host batches in either of two forms:

* ``(images [B, ...], labels [B])`` (a ``DataLoader``): the images cross PCIe
  in their own dtype and layout, and on the copy stream they are transposed
  to the trainer's feature-major input ``x [features, B]`` and cast, while
  the labels become the one-hot target ``y [C, B]``;
* ``(x [features, B], y [C, B])`` already in the trainer's layout and dtype:
  copied as they are.

A batch that is not in pinned memory is first written into a pinned staging
buffer of its slot (a host memcpy); pinned batches are copied from directly
and kept referenced until their copy is done.  ``next()`` makes the caller's
current stream wait for that slot's copy and returns its device tensors; a
slot is refilled only after the compute stream has passed the point where the
caller handed it back (the next ``next()`` call, or ``release()``).

``steps_per_slot > 1`` groups that many consecutive batches into one slot as a
pool ``x [S, features, B]``, ``y [S, C, B]`` -- the operand layout of
``TileLangIPC.train_pool``, which trains on all of them in one
persistent-kernel launch.  A source may also yield such pools itself
(``x [S, features, B]``, ``y [S, C, B]``, S <= ``steps_per_slot``): each
fills one slot with a single copy per tensor.
"""
from __future__ import annotations

from typing import Iterable, Iterator

import torch


class BatchPipeline:
    def __init__(self, source: Iterable, *, device: torch.device, dtype: torch.dtype, num_classes: int,
                 depth: int = 2, steps_per_slot: int = 1):
        if depth < 2:
            raise ValueError("depth must be >= 2 (one slot in use, one being filled)")
        if steps_per_slot < 1:
            raise ValueError("steps_per_slot must be >= 1")
        self.device = torch.device(device)
        self.dtype = dtype
        self.num_classes = int(num_classes)
        self.depth = int(depth)
        self.per_slot = int(steps_per_slot)
        self._it: Iterator = iter(source)
        self._copy = torch.cuda.Stream(self.device)
        self._slots: list[dict | None] = [None] * self.depth
        self._ready = [torch.cuda.Event() for _ in range(self.depth)]
        self._free = [torch.cuda.Event() for _ in range(self.depth)]
        self._copied = [torch.cuda.Event() for _ in range(self.depth)]  # staging of the slot read by its H2D
        self._count = [0] * self.depth
        self._head = 0                  # next slot handed out
        self._out: int | None = None    # slot currently held by the caller
        self._exhausted = False
        self.h2d_bytes = 0              # host -> device bytes issued so far
        for k in range(self.depth):
            self._fill(k)

    # ------------------------------------------------------------------ slots
    def _alloc(self, a: torch.Tensor, b: torch.Tensor) -> dict:
        S, dev = self.per_slot, self.device
        if b.ndim == 1:  # images + labels
            B, F = int(a.shape[0]), int(a[0].numel())
            return {"kind": "images", "key": ("images", B, F, a.dtype),
                    "a_h": None, "b_h": None, "h_shapes": ((S, B, F), a.dtype, (S, B), torch.int64),
                    "a_d": torch.empty((S, B, F), dtype=a.dtype, device=dev),
                    "b_d": torch.empty((S, B), dtype=torch.int64, device=dev),
                    "x": torch.empty((S, F, B), dtype=self.dtype, device=dev),
                    "y": torch.zeros((S, self.num_classes, B), dtype=self.dtype, device=dev)}
        F, B = int(a.shape[-2]), int(a.shape[-1])
        x = torch.empty((S, F, B), dtype=self.dtype, device=dev)
        y = torch.empty((S, self.num_classes, B), dtype=self.dtype, device=dev)
        return {"kind": "prepared", "key": ("prepared", B, F, a.dtype),
                "a_h": None, "b_h": None,
                "h_shapes": ((S, F, B), self.dtype, (S, self.num_classes, B), self.dtype),
                "a_d": x, "b_d": y, "x": x, "y": y}

    @staticmethod
    def _staging(slot: dict) -> None:
        """The slot's pinned staging buffers, allocated on first need (pinned sources never need them)."""
        if slot["a_h"] is None:
            sa, da, sb, db = slot["h_shapes"]
            slot["a_h"] = torch.empty(sa, dtype=da).pin_memory()
            slot["b_h"] = torch.empty(sb, dtype=db).pin_memory()

    def _take(self) -> list:
        """The host items of the next slot: ``per_slot`` batches, or one pool chunk (3-D x and y)."""
        items = []
        while not self._exhausted:
            try:
                a, b = next(self._it)
            except StopIteration:
                self._exhausted = True
                break
            if b.ndim == 3:  # a pool chunk [S, d, B] fills a slot by itself
                if items:
                    raise ValueError("pool chunks and single batches cannot be mixed in one pipeline")
                if a.ndim != 3 or a.shape[0] != b.shape[0] or not 1 <= a.shape[0] <= self.per_slot:
                    raise ValueError("a pool chunk is x [S, features, B], y [S, C, B] with 1 <= S <= steps_per_slot")
                return [(a, b)]
            items.append((a, b))
            if len(items) == self.per_slot:
                break
        return items

    def _fill(self, k: int) -> None:
        """Queue the copy of the next slot's host batches into slot k on the copy stream."""
        items = self._take()
        self._count[k] = 0
        if not items:
            return
        a0, b0 = items[0]
        if b0.ndim == 1:
            key = ("images", int(a0.shape[0]), int(a0[0].numel()), a0.dtype)
        else:
            if a0.ndim != b0.ndim or a0.shape[-1] != b0.shape[-1] or b0.shape[-2] != self.num_classes:
                raise ValueError("prepared batches must be x [features, B] and y [num_classes, B]")
            key = ("prepared", int(a0.shape[-1]), int(a0.shape[-2]), self.dtype)
        slot = self._slots[k]
        if slot is None or slot["key"] != key:
            slot = self._slots[k] = self._alloc(a0, b0)
        self._copied[k].synchronize()  # the previous copy out of this slot's staging buffers is done
        pool = b0.ndim == 3
        n = int(a0.shape[0]) if pool else len(items)
        srcs = []
        sa, _, sb, _ = slot["h_shapes"]
        for j, (a, b) in enumerate(items):
            if slot["kind"] == "images":
                a = a.reshape(a.shape[0], -1)
                if tuple(a.shape) != tuple(sa[1:]) or tuple(b.shape) != (sa[1],):
                    raise ValueError("every batch of a pipeline must have the same shape")
                b = b.to(torch.int64)
            else:
                if tuple(a.shape[-2:]) != tuple(sa[1:]) or tuple(b.shape[-2:]) != tuple(sb[1:]):
                    raise ValueError("every batch of a pipeline must have the same shape")
                if a.dtype != self.dtype or b.dtype != self.dtype:
                    raise ValueError("prepared batches must already be in the pipeline dtype")
            if not (a.is_pinned() and a.is_contiguous()):
                self._staging(slot)
                dst_a = slot["a_h"][:n] if pool else slot["a_h"][j]
                dst_a.copy_(a)
                a = dst_a
            if not (b.is_pinned() and b.is_contiguous()):
                self._staging(slot)
                dst_b = slot["b_h"][:n] if pool else slot["b_h"][j]
                dst_b.copy_(b)
                b = dst_b
            srcs.append((a, b))
        with torch.cuda.stream(self._copy):
            self._copy.wait_event(self._free[k])  # the compute stream is done with this slot
            for j, (a, b) in enumerate(srcs):
                (slot["a_d"][:n] if pool else slot["a_d"][j]).copy_(a, non_blocking=True)
                (slot["b_d"][:n] if pool else slot["b_d"][j]).copy_(b, non_blocking=True)
                self.h2d_bytes += a.numel() * a.element_size() + b.numel() * b.element_size()
            self._copied[k].record(self._copy)
            if slot["kind"] == "images":
                slot["x"][:n].copy_(slot["a_d"][:n].transpose(1, 2))
                slot["y"][:n].zero_()
                slot["y"][:n].scatter_(1, slot["b_d"][:n].unsqueeze(1), 1.0)
            self._ready[k].record(self._copy)
        slot["sources"] = srcs  # pinned sources stay referenced until their copies are done
        self._count[k] = n

    # ------------------------------------------------------------- consumer
    def release(self) -> None:
        """Hand the current slot back; its refill waits for the work queued so far on the current stream."""
        if self._out is None:
            return
        k, self._out = self._out, None
        self._free[k].record(torch.cuda.current_stream(self.device))
        self._fill(k)

    def next(self) -> tuple[torch.Tensor, torch.Tensor] | None:
        """The next batch (or pool of ``steps_per_slot`` batches) on the device, ready on the current
        stream: ``(x, y)`` of shapes ``[features, B]`` / ``[C, B]`` (a pool: with a leading batch
        count, which is below ``steps_per_slot`` only for the last, partial pool).  ``None`` when the
        source is exhausted."""
        self.release()
        k = self._head
        n = self._count[k]
        if n == 0:
            return None
        self._head = (k + 1) % self.depth
        self._out = k
        torch.cuda.current_stream(self.device).wait_event(self._ready[k])
        slot = self._slots[k]
        if self.per_slot == 1:
            return slot["x"][0], slot["y"][0]
        return slot["x"][:n], slot["y"][:n]

    def __iter__(self):
        while True:
            b = self.next()
            if b is None:
                return
            yield b
