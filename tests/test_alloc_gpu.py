"""Device block cache behind fz_malloc / fz_free (the role of Fusion's PoolAllocator,
fusion/src/Fusion/alloc/BFCPoolAllocator.cpp:59-111, and its tests in
fusion/tests/alloc): a freed block is reused by the next allocation of its size
class on the same stream, never by another stream, accounting follows the blocks,
and a pointer the allocator did not hand out is refused."""
import ctypes as C
import threading

import pytest

pytestmark = pytest.mark.gpu


def _stats(L):
    r, u = C.c_size_t(), C.c_size_t()
    assert L.fz_pool_stats(C.byref(r), C.byref(u)) == 0
    return r.value, u.value


def _alloc(capi, n, stream=None):
    p = C.c_void_p()
    capi.check(capi.lib().fz_malloc(C.byref(p), n, stream))
    return p.value


def test_freed_block_is_reused_on_same_stream(capi):
    L = capi.lib()
    a = _alloc(capi, 3 << 20)
    capi.check(L.fz_free(a, None))
    b = _alloc(capi, (3 << 20) - 1000)  # same 2 MiB size class
    assert b == a
    c = _alloc(capi, 3 << 20)  # a second live block of the class is a new block
    assert c != b
    capi.check(L.fz_free(b, None))
    capi.check(L.fz_free(c, None))


def test_size_classes_keep_blocks_apart(capi):
    L = capi.lib()
    a = _alloc(capi, 1000)
    capi.check(L.fz_free(a, None))
    b = _alloc(capi, 5000)  # another 512 B class: not the cached block
    assert b != a
    capi.check(L.fz_free(b, None))
    assert _alloc(capi, 600) == a  # 600 and 1000 share the 1024 B class
    capi.check(L.fz_free(a, None))


def test_other_stream_does_not_take_cached_block(capi):
    L = capi.lib()
    a = _alloc(capi, 7 << 20)
    capi.check(L.fz_free(a, None))
    got = {}

    def other():  # another thread has its own per-thread stream
        capi.check(L.fz_set_device(0))
        got["p"] = _alloc(capi, 7 << 20)
        capi.check(L.fz_stream_sync(None))

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert got["p"] != a
    assert _alloc(capi, 7 << 20) == a
    capi.check(L.fz_free(a, None))
    capi.check(L.fz_free(got["p"], None))


def test_used_bytes_follow_blocks_and_release(capi):
    L = capi.lib()
    capi.check(L.fz_stream_sync(None))
    _, u0 = _stats(L)
    a = _alloc(capi, 64 << 20)
    _, u1 = _stats(L)
    assert u1 - u0 == 64 << 20
    capi.check(L.fz_free(a, None))
    r2, u2 = _stats(L)
    assert u2 == u0
    capi.check(L.fz_pool_release())
    r3, u3 = _stats(L)
    assert u3 == u0 and r3 <= r2


def test_free_of_foreign_pointer_is_refused(capi):
    L = capi.lib()
    a = _alloc(capi, 4096)
    capi.check(L.fz_free(a, None))
    assert L.fz_free(a, None) == 1  # FZ_ERR_INVALID: freed twice
    assert b"fz_malloc" in L.fz_last_error()
    assert L.fz_free(C.c_void_p(a + 512), None) == 1


def test_data_survives_reuse_in_stream_order(capi):
    """A block freed while a copy into it is still queued is reused only after it."""
    import numpy as np

    L = capi.lib()
    n = 1 << 22
    x = np.arange(n, dtype=np.float32)
    for _ in range(3):
        d = capi.DeviceArray.from_numpy(x)
        y = capi.DeviceArray((n,))
        capi.check(L.fz_memcpy_d2d(y.ptr, d.ptr, x.nbytes, None))
        del d  # freed on the stream; the next from_numpy may take the same block
        z = capi.DeviceArray.from_numpy(np.zeros(n, np.float32))
        np.testing.assert_array_equal(y.numpy(), x)
        del y, z


def test_block_freed_on_another_stream_returns_home_after_its_use(capi):
    """A block allocated on the upload stream and freed on the compute stream goes back
    to the upload stream's cache. It is handed out there again only once the compute
    stream has passed the free; before that a request takes other memory, so a write on
    the upload stream never lands under the queued reads."""
    import numpy as np

    L = capi.lib()
    L.fz_upload_stream.restype = C.c_void_p
    up = C.c_void_p(L.fz_upload_stream())
    n = 1 << 22
    x = np.arange(n, dtype=np.float32)
    p = C.c_void_p()
    capi.check(L.fz_malloc(C.byref(p), n * 4, up))
    capi.check(L.fz_memcpy_h2d(p, x.ctypes.data, n * 4, up))
    capi.check(L.fz_stream_wait(None, up))
    q = capi.DeviceArray((n,))
    for _ in range(8):  # queue compute-stream reads of the block
        capi.check(L.fz_memcpy_d2d(q.ptr, p, n * 4, None))
    capi.check(L.fz_free(p, None))  # freed on the compute stream
    p2 = C.c_void_p()
    capi.check(L.fz_malloc(C.byref(p2), n * 4, up))
    z = np.zeros(n, np.float32)
    capi.check(L.fz_memcpy_h2d(p2, z.ctypes.data, n * 4, up))
    capi.check(L.fz_stream_sync(up))
    np.testing.assert_array_equal(q.numpy(), x)  # the queued reads saw the old contents
    capi.check(L.fz_free(p2, up))
    capi.check(L.fz_stream_sync(None))  # the compute stream is past the free now
    p3, p4 = C.c_void_p(), C.c_void_p()
    capi.check(L.fz_malloc(C.byref(p3), n * 4, up))
    capi.check(L.fz_malloc(C.byref(p4), n * 4, up))
    assert p.value in (p3.value, p4.value)  # back in its home cache
    capi.check(L.fz_free(p3, up))
    capi.check(L.fz_free(p4, up))


def test_stream_destroy_returns_its_cached_blocks(capi):
    """Blocks cached for a stream leave the cache when the stream is destroyed (a new
    stream may get the same handle), and a block still live on it is re-homed: freeing
    it afterwards caches it for the thread's compute stream, where it is reused."""
    L = capi.lib()
    L.fz_pool_cached.argtypes = [C.POINTER(C.c_size_t)]

    def cached():
        v = C.c_size_t()
        capi.check(L.fz_pool_cached(C.byref(v)))
        return v.value

    s = C.c_void_p()
    capi.check(L.fz_stream_create(C.byref(s)))
    p, keep = C.c_void_p(), C.c_void_p()
    capi.check(L.fz_malloc(C.byref(p), 3 << 20, s))
    capi.check(L.fz_malloc(C.byref(keep), 5 << 20, s))
    c0 = cached()
    capi.check(L.fz_free(p, s))
    assert cached() == c0 + (4 << 20)  # 2 MiB size classes above 1 MiB
    capi.check(L.fz_stream_destroy(s))
    assert cached() == c0
    capi.check(L.fz_stream_sync(None))
    capi.check(L.fz_free(keep, None))  # live block of the destroyed stream
    assert cached() == c0 + (6 << 20)
    q = C.c_void_p()
    capi.check(L.fz_malloc(C.byref(q), 5 << 20, None))
    assert q.value == keep.value  # reused from the compute stream's cache
    capi.check(L.fz_free(q, None))
    s2 = C.c_void_p()
    capi.check(L.fz_stream_create(C.byref(s2)))
    r = C.c_void_p()
    capi.check(L.fz_malloc(C.byref(r), 3 << 20, s2))  # nothing stale cached for s2
    capi.check(L.fz_free(r, s2))
    capi.check(L.fz_stream_destroy(s2))
