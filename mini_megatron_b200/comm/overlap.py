"""Communication/compute overlap helpers with correct stream fencing.

Reference: comm/overlap_tp.py:6-26 and comm/overlap_pp.py:5-27.  The
reference launches the collective on a side stream without making that
stream wait for the producer of the tensor (a race).  Here the side stream
first waits on the current stream, the tensor is marked as used by the side
stream (so the caching allocator does not recycle it early), and
``synchronize`` makes the *current stream* wait on the side stream instead of
blocking the host.
"""
import torch
import torch.distributed as dist


class _SideStream:
    def __init__(self):
        self.stream = torch.cuda.Stream() if torch.cuda.is_available() else None

    def enter(self, tensor):
        if self.stream is None:
            return None
        cur = torch.cuda.current_stream()
        self.stream.wait_stream(cur)
        tensor.record_stream(self.stream)
        return torch.cuda.stream(self.stream)


class AsyncAllReduce(_SideStream):
    """Launch ``all_reduce(tensor)`` off the critical path; ``synchronize()`` joins it."""

    def __init__(self, group):
        super().__init__()
        self.group = group
        self.pending = []

    def all_reduce_async(self, tensor):
        if self.group is None or dist.get_world_size(self.group) == 1:
            return tensor
        ctx = self.enter(tensor)
        if ctx is None:
            work = dist.all_reduce(tensor, group=self.group, async_op=True)
            self.pending.append(work)
            return tensor
        with ctx:
            dist.all_reduce(tensor, group=self.group)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self.pending.append(ev)
        return tensor

    def synchronize(self):
        for item in self.pending:
            if isinstance(item, torch.cuda.Event):
                torch.cuda.current_stream().wait_event(item)
            else:
                item.wait()
        self.pending.clear()


class AsyncP2P(_SideStream):
    """Non-blocking isend/irecv on a side stream, fenced against the producer."""

    def __init__(self, group=None):
        super().__init__()
        self.group = group
        self.requests = []

    def send_async(self, tensor, dst):
        ctx = self.enter(tensor)
        if ctx is None:
            self.requests.append((dist.isend(tensor, dst=dst, group=self.group), tensor))
            return
        with ctx:
            self.requests.append((dist.isend(tensor, dst=dst, group=self.group), tensor))

    def recv_async(self, tensor, src):
        ctx = self.enter(tensor)
        if ctx is None:
            self.requests.append((dist.irecv(tensor, src=src, group=self.group), tensor))
            return tensor
        with ctx:
            self.requests.append((dist.irecv(tensor, src=src, group=self.group), tensor))
        return tensor

    def synchronize(self):
        for req, _ in self.requests:
            req.wait()
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)
        self.requests.clear()
