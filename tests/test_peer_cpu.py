"""Host-side checks of the peer-memory collective API without a GPU: the
argument and state errors of lmpb_peer_import / lmpb_reduce_allreduce come
back as LMPB_ERR_INVALID with a message before any CUDA call, and no peer
context exists until one is imported."""
from __future__ import annotations

import ctypes as C

from rushlite_b200 import capi


def test_no_context_until_imported():
    assert capi.peer_size() == 0
    shape = (C.c_int64 * 2)(4096, 4096)
    st = capi.lib().lmpb_reduce_allreduce(capi.SUM, capi.FLOAT32, None, shape, 2, 0, None, None)
    assert st == 1 and b"no peer context" in capi.lib().lmpb_last_error()


def test_import_rejects_bad_arguments():
    L = capi.lib()
    h = C.create_string_buffer(capi.PEER_HANDLE_BYTES * 2)
    assert L.lmpb_peer_import(None, 2, 0) == 1
    assert L.lmpb_peer_import(h, 9, 0) == 1          # more ranks than the context holds
    assert L.lmpb_peer_import(h, 2, 2) == 1          # rank outside [0, nranks)
    assert L.lmpb_peer_import(h, 2, 0) == 1          # nothing exported yet
    assert b"lmpb_peer_export first" in L.lmpb_last_error()
    assert L.lmpb_peer_export(h, 8) == 1             # handle buffer too small
    assert capi.peer_size() == 0
