"""Host-resident data through the device ops with the transfers overlapped.

A checkpoint being quantized, or a batch of activations, often lives in host
memory: it reaches the quantizers over PCIe and the results go back the same
way.  Item by item on one stream, the host->device copy, the kernels and the
device->host copy run one after another.  PCIe is full duplex and the copy
engines work beside the SMs, so ``HostPipeline`` puts the three on their own
CUDA streams: the upload of item i+1, the work on item i and the download of
item i-1 overlap, and a sequence costs about its largest transfer instead of
the sum of all three.

The reference (qlora.py, core/quantizer.py, kv_cache_quant.py) has no
counterpart: its torch code runs wherever its tensors are.
"""

from __future__ import annotations

from typing import Callable, Dict, Optional

import torch


class HostPipeline:
    """Three CUDA streams (upload, work, download) with the ordering a
    pipelined host round trip needs.

    ``run(n, upload, work, download)`` calls, for i = 0 .. n-1,

    * ``upload(i, buf)`` on the upload stream, ``buf = i % buffers``: copy
      item i from (pinned) host memory into device input buffer ``buf``.  It
      waits until the work that last read that buffer has finished.
    * ``work(i, buf)`` on the work stream, after upload(i): the device ops
      (library calls launch on the current stream, which is the work stream).
      With ``outputs_reused=True`` it also waits for the previous run's
      download of item i, for work that rewrites the same output buffers
      every run (a replayed CUDA graph).
    * ``download(i, buf)`` on the download stream, after work(i): copy the
      results to (pinned) host memory.  A tensor that work(i) allocated and
      download(i) reads must stay allocated until the copy has run: call
      ``t.record_stream(torch.cuda.current_stream())`` on it in download.

    The calling stream waits for all three streams before ``run`` returns,
    so CUDA events recorded on it around ``run`` time the whole sequence;
    host buffers are safe to read after synchronizing that stream.  The
    ordering state persists across runs of the same object.
    """

    def __init__(self, device: Optional[torch.device] = None, buffers: int = 2):
        if buffers < 1:
            raise ValueError("buffers must be >= 1")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        self.buffers = buffers
        self.up = torch.cuda.Stream(self.device)
        self.work = torch.cuda.Stream(self.device)
        self.down = torch.cuda.Stream(self.device)
        self._worked: Dict[int, torch.cuda.Event] = {}  # input buffer -> last work that read it
        self._stored: Dict[int, torch.cuda.Event] = {}  # item -> its last download

    def run(self, n: int, upload: Callable[[int, int], None], work: Callable[[int, int], None],
            download: Callable[[int, int], None], outputs_reused: bool = False) -> None:
        cur = torch.cuda.current_stream(self.device)
        for s in (self.up, self.work, self.down):
            s.wait_stream(cur)
        for i in range(n):
            buf = i % self.buffers
            with torch.cuda.stream(self.up):
                prev = self._worked.get(buf)
                if prev is not None:
                    self.up.wait_event(prev)
                upload(i, buf)
                loaded = torch.cuda.Event()
                loaded.record(self.up)
            with torch.cuda.stream(self.work):
                self.work.wait_event(loaded)
                if outputs_reused and i in self._stored:
                    self.work.wait_event(self._stored[i])
                work(i, buf)
                done = torch.cuda.Event()
                done.record(self.work)
                self._worked[buf] = done
            with torch.cuda.stream(self.down):
                self.down.wait_event(done)
                download(i, buf)
                stored = torch.cuda.Event()
                stored.record(self.down)
                self._stored[i] = stored
        for s in (self.up, self.work, self.down):
            cur.wait_stream(s)
