"""Bounded peer wait of the fused all-reduce GEMV (tf_w4a16_linear_allreduce) running out, on one
GPU and without a fault.

A world-2 peer set is built whose "peer" mailbox is a second local buffer: rank 0's kernel
stores its partials there and then polls its own mailbox for rank 1's values, which nothing
ever writes. Every poll must give up after the kernel's 2 s limit, record the time-out in the
mailbox's error word and return; the host reads the word with tf_peer_mailbox_error (which
clears it), and the context stays usable for the next launch.
"""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

from oracle import oracle
from tests.numerics import cases
from tests.numerics.tolerance import atol
import tokenforge_b200.ops  # noqa: F401  (registers torch.ops.tokenforge)
from tokenforge_b200 import _lib

pytestmark = pytest.mark.gpu
G = 128


def _weights(n: int, k: int, device: torch.device):
    qweight, qzeros, scales = cases.random_awq(n, k, 5)
    qt = oracle.repack_awq_to_tf(qweight)
    return qt.to(device), scales.to(device), qzeros.to(device), oracle.dequantize_tf(
        qt, scales, qzeros, G)


def test_silent_peer_times_out_and_reports(device: torch.device) -> None:
    lib = _lib.lib()
    n, k = 256, 1024
    qt, s, z, w16 = _weights(n, k, device)
    x = cases.activations(1, k, 9).to(device)
    y = torch.full((1, n), float("nan"), dtype=torch.float16, device=device)
    nbytes = int(lib.tf_peer_mailbox_bytes(2, 1, n))
    own, fake = ctypes.c_void_p(), ctypes.c_void_p()
    handle = (ctypes.c_char * _lib.TF_IPC_HANDLE_BYTES)()
    with torch.cuda.device(device):
        _lib.check("tf_peer_mailbox_alloc", lib.tf_peer_mailbox_alloc(nbytes, ctypes.byref(own), handle))
        _lib.check("tf_peer_mailbox_alloc", lib.tf_peer_mailbox_alloc(nbytes, ctypes.byref(fake), handle))
    try:
        peers = _lib.TfPeerSet()
        peers.rank, peers.world, peers.max_m, peers.max_n = 0, 2, 1, n
        peers.mailbox[0], peers.mailbox[1] = own.value, fake.value
        torch.cuda.synchronize(device)
        t0 = time.monotonic()
        with torch.cuda.device(device):
            st = lib.tf_w4a16_linear_allreduce(
                x.data_ptr(), 1, k, k, qt.data_ptr(), s.data_ptr(), z.data_ptr(), None, n, G,
                y.data_ptr(), n, None, 0, ctypes.byref(peers), _lib.stream_ptr(device))
        _lib.check("tf_w4a16_linear_allreduce", st)
        torch.cuda.synchronize(device)
        waited = time.monotonic() - t0
        assert 1.5 <= waited <= 30.0, f"kernel returned after {waited:.2f} s"
        code = ctypes.c_int(0)
        _lib.check("tf_peer_mailbox_error", lib.tf_peer_mailbox_error(own, ctypes.byref(code)))
        assert code.value != 0, "the time-out was not recorded"
        _lib.check("tf_peer_mailbox_error", lib.tf_peer_mailbox_error(own, ctypes.byref(code)))
        assert code.value == 0, "reading the error word clears it"
        # The context is intact: an ordinary launch afterwards is correct.
        y2 = torch.ops.tokenforge.w4a16_linear(x, qt, s, z, None, G, "cuda")
        ref = x.double().cpu() @ w16.double().t()
        err = float((y2.double().cpu() - ref).abs().max())
        assert err <= atol(x.cpu(), w16, "cuda")
    finally:
        torch.cuda.synchronize(device)
        with torch.cuda.device(device):
            _lib.check("tf_peer_mailbox_free", lib.tf_peer_mailbox_free(own))
            _lib.check("tf_peer_mailbox_free", lib.tf_peer_mailbox_free(fake))
