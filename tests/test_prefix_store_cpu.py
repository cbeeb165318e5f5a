"""The native persistent prefix store on the CPU: round trips, persistence across
reopen, torn manifest tails, corrupt data (checksum -> miss, never wrong bytes)
and the capacity bound.

Mirrors the reference's prefix-cache fault checks: a flipped byte must make the
reader fall back to recompute (scripts/runtime/glm53-prefix-cache-fault.sh:1-45)
and a torn tail is recovered on open (engines/glm5-moe-nvfp4-2b/src/kv/
nvme_prefix_store.cc:389-480).
"""
import os

import numpy as np
import pytest

from rocket_b200 import _rt


def _parts(seed, sizes=(1000, 70000, 13)):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, n, dtype=np.uint8) for n in sizes]


def _get(st, k, fp=7):
    r = st.get(k, fp)
    return None if r is None else [np.frombuffer(b, dtype=np.uint8) for b in r]


def test_round_trip_and_reopen(tmp_path):
    d = str(tmp_path)
    st = _rt.PrefixStore(d, 1 << 30)
    for k in range(5):
        assert st.put(k + 100, 7, _parts(k))
    assert not st.put(100, 7, _parts(0))  # exists
    assert st.contains(102, 7) and not st.contains(102, 8)
    got = _get(st, 103)
    assert all(np.array_equal(a, b) for a, b in zip(got, _parts(3)))
    del st
    st2 = _rt.PrefixStore(d, 1 << 30)
    assert st2.stats()["live_records"] == 5
    got = _get(st2, 104)
    assert all(np.array_equal(a, b) for a, b in zip(got, _parts(4)))
    # get_into fills caller buffers
    outs = [np.zeros(n, dtype=np.uint8) for n in st2.sizes(101, 7)]
    assert st2.get_into(101, 7, outs)
    assert all(np.array_equal(a, b) for a, b in zip(outs, _parts(1)))


@pytest.mark.parametrize("cut", [1, 60, 143])
def test_torn_manifest_tail_is_recovered(tmp_path, cut):
    d = str(tmp_path)
    st = _rt.PrefixStore(d, 1 << 30)
    for k in range(3):
        st.put(k, 7, _parts(k))
    del st
    man = os.path.join(d, "manifest.bin")
    size = os.path.getsize(man)
    with open(man, "r+b") as f:  # a crash in the middle of the 4th manifest append
        f.seek(size)
        f.write(b"\x4d\x54\x4b\x52" + b"\x01" * (cut - 4 if cut > 4 else 0))
    st = _rt.PrefixStore(d, 1 << 30)
    s = st.stats()
    assert s["torn_tail_recoveries"] == 1 and s["live_records"] == 3
    assert os.path.getsize(man) == size
    assert all(np.array_equal(a, b) for a, b in zip(_get(st, 2), _parts(2)))
    assert st.put(9, 7, _parts(9))  # appends continue after recovery
    del st
    assert _rt.PrefixStore(d, 1 << 30).stats()["live_records"] == 4


def test_flipped_byte_reads_as_miss(tmp_path):
    d = str(tmp_path)
    st = _rt.PrefixStore(d, 1 << 30)
    st.put(1, 7, _parts(1))
    st.put(2, 7, _parts(2))
    del st
    seg = os.path.join(d, "segments", sorted(os.listdir(os.path.join(d, "segments")))[0])
    with open(seg, "r+b") as f:
        f.seek(500)  # inside record 1's first component
        b = f.read(1)
        f.seek(500)
        f.write(bytes([b[0] ^ 0x10]))
    st = _rt.PrefixStore(d, 1 << 30)
    assert _get(st, 1) is None
    s = st.stats()
    assert s["checksum_failures"] == 1 and not st.contains(1, 7)
    assert all(np.array_equal(a, b) for a, b in zip(_get(st, 2), _parts(2)))
    del st
    assert not _rt.PrefixStore(d, 1 << 30).contains(1, 7)  # the drop is persistent


def test_capacity_evicts_oldest_segments(tmp_path):
    d = str(tmp_path)
    st = _rt.PrefixStore(d, 4 << 20, segment_bytes=1 << 20)
    for k in range(40):
        st.put(k, 7, _parts(k, sizes=(200000,)))
    s = st.stats()
    assert s["evicted_records"] > 0
    assert s["live_bytes"] <= 4 << 20
    assert st.contains(39, 7) and not st.contains(0, 7)
    assert len(os.listdir(os.path.join(d, "segments"))) <= 5


def test_random_operations_against_a_model(tmp_path):
    """Property test: random put / erase / get / reopen sequences under a small capacity.
    A read returns either the exact bytes last put under that key or a miss (capacity
    eviction) -- never other bytes -- and erased keys stay gone, also across reopens."""
    import random
    d = str(tmp_path)
    rng = random.Random(7)
    cap = 1 << 20
    st = _rt.PrefixStore(d, cap, 256 << 10, False)
    model = {}           # key -> parts last put (may have been evicted since)
    erased = set()
    for step in range(300):
        op = rng.choice(["put", "put", "get", "get", "erase", "reopen"])
        key = rng.randrange(40)
        if op == "put":
            parts = _parts(step, sizes=(rng.randint(1, 30000), rng.randint(0, 5000)))
            if st.put(key, 7, parts):
                model[key] = parts
                erased.discard(key)
        elif op == "get":
            got = _get(st, key)
            if got is not None:
                assert key in model and key not in erased, key
                assert all(np.array_equal(a, b) for a, b in zip(got, model[key])), key
        elif op == "erase":
            st.erase(key, 7)
            model.pop(key, None)
            erased.add(key)
            assert _get(st, key) is None
        else:
            st.flush()
            del st
            st = _rt.PrefixStore(d, cap, 256 << 10, False)
        s = st.stats()
        assert s["checksum_failures"] == 0


def test_free_space_headroom_skips_puts(tmp_path):
    import shutil

    import numpy as np
    from rocket_b200 import _rt
    st = _rt.PrefixStore(str(tmp_path), 1 << 30)
    assert st.min_free_bytes() == 256 << 20
    st.set_min_free_bytes(shutil.disk_usage(str(tmp_path)).free + (1 << 40))  # more than the disk has
    part = np.arange(1000, dtype=np.uint8)
    assert not st.put(1, 2, [part])
    assert st.stats()["refused_low_space"] == 1 and not st.contains(1, 2)
    st.set_min_free_bytes(0)
    assert st.put(1, 2, [part]) and st.contains(1, 2)
