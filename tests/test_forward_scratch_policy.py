"""CPU: which forward paths may allocate key-split scratch.

The reference's ``_launch_forward`` (and the registry launchers built on it)
writes into caller buffers and allocates nothing; this package keeps that
contract, so those paths never take the key-split schedule.  The public
``attention_*`` calls and the autograd forward allocate their outputs anyway
and do take it for problems too small to fill the GPU.  The library is
replaced by a recording stand-in, so no GPU is needed: the test checks what
the Python layer asks the C ABI for, not the kernels.
"""

from __future__ import annotations

import contextlib

import pytest
import torch

from tklab.kernels import flash_attention as fa


class _RecordingLib:
    """Stands in for libtklab_attn.so: records the forward calls it receives."""

    def __init__(self, ws_bytes: int) -> None:
        self.ws_bytes = ws_bytes
        self.size_queries = 0
        self.calls: list[tuple[object, int]] = []

    def tk_attn_fwd_workspace_bytes(self, *args) -> int:
        self.size_queries += 1
        return self.ws_bytes

    def tk_attn_fwd_ws(self, *args) -> int:
        workspace, ws_bytes = args[12], args[13]
        self.calls.append((workspace, ws_bytes))
        return 0


@pytest.fixture()
def recording(monkeypatch):
    lib = _RecordingLib(ws_bytes=4096)
    monkeypatch.setattr(fa._native, "load", lambda: lib)
    monkeypatch.setattr(fa, "_on_device", lambda device: contextlib.nullcontext())
    monkeypatch.setattr(fa, "_stream", lambda tensor: 0)
    monkeypatch.setattr(fa, "_after_launch", lambda device: None)
    fa._forward_workspace_bytes.cache_clear()
    yield lib
    fa._forward_workspace_bytes.cache_clear()


def _qkv():
    return [torch.zeros((1, 2, 8192, 128), dtype=torch.bfloat16) for _ in range(3)]


def test_caller_buffer_launch_allocates_nothing(recording) -> None:
    q, k, v = _qkv()
    out = torch.empty_like(q)
    fa._forward_checked(q, k, v, out, out, causal=True, store_lse=False)
    assert recording.calls == [(None, 0)]
    assert recording.size_queries == 0


def test_allocating_paths_pass_key_split_scratch(recording) -> None:
    q, k, v = _qkv()
    out = torch.empty_like(q)
    fa._forward_launch(q, k, v, out, None, causal=True, key_split=True)
    (workspace, ws_bytes), = recording.calls
    assert workspace is not None and ws_bytes == 4096
    assert recording.size_queries == 1


def test_no_scratch_when_the_problem_fills_the_device(recording) -> None:
    recording.ws_bytes = 0
    q, k, v = _qkv()
    out = torch.empty_like(q)
    fa._forward_launch(q, k, v, out, None, causal=False, key_split=True)
    assert recording.calls == [(None, 0)]
