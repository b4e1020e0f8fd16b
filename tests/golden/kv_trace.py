"""Record and replay of the calls the reference's KVCacheManager makes into
``matmul_module`` — TEST INFRASTRUCTURE.

The reference's ``src/kv_cache.py`` is the drop-in boundary's caller: it stays
unchanged and reaches the KV path only through ``matmul_module.kv_cache_init``,
``kv_cache_free``, ``gqa_attention_cached`` (gpu mode, kv_cache.py:240-256) and
``gqa_attention`` (cpu / mmap modes, kv_cache.py:219-239, called with the
layer's view of its host arrays after the host append).  The reference is not
available where the GPU tests run, so ``make_kv_trace.py`` runs it here with a
``Recorder`` in place of ``matmul_module`` and stores what crossed the
boundary: every call with its scalar arguments; every array argument either as
its contents or, for views of the manager's host arrays, as (host array,
layer); the host arrays' creation (numpy array or memory-mapped file, shape)
and every change the manager made to their contents between calls; and the
expected output of each attention call from the reference's numpy oracle.

``replay`` performs the same sequence against a module (the shim
``matmul_module`` in the GPU tests): it builds host arrays of the same kind,
applies the recorded writes, passes the same views, and returns every call's
output and any exception.  The host arrays are released where the manager
released them (close()).
"""

from __future__ import annotations

import json
import mmap
import os
import tempfile

import numpy as np

TRACE_FILE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kv_trace.npz")


def _owner(a):
    o = a
    while isinstance(o.base, np.ndarray):
        o = o.base
    return o


class Recorder:
    """Stand-in for ``matmul_module`` while the reference's KVCacheManager runs.

    ``ref(Q, K, V, start_pos, scale, causal)`` computes an expected output (the
    reference's ``ref_gqa_attention``); the gpu-mode pool is modelled by a host
    array with the semantics of launch_gqa_attention_cached_fp16
    (attention.hip:302-374: rows written at start_pos, attention over
    [0, start_pos + q_len))."""

    def __init__(self, ref):
        self.ref = ref
        self.events = []
        self.arrays = {}
        self._owners = {}      # id(owner) -> (index, weak reference, shadow copy)
        self._pool = None
        self.fail_init = False

    # -- storage -------------------------------------------------------------
    def _store(self, a) -> str:
        name = f"a{len(self.arrays)}"
        self.arrays[name] = np.array(a, copy=True)
        return name

    def _sync_owner(self, o, lo_hi):
        """Register a host array (first use) and record what changed in its
        elements [lo, hi) (the rows the call reads) since they were last recorded."""
        import weakref

        key = id(o)
        if key not in self._owners or self._owners[key][1]() is not o:
            j = len(self._owners)
            kind = "mmap" if isinstance(o.base, (memoryview, mmap.mmap)) else "ndarray"
            self.events.append({"op": "host", "id": j, "kind": kind, "size": int(o.size),
                                "dtype": str(o.dtype)})
            shadow = np.zeros(o.size, o.dtype)
            # weak references only: the manager must be able to close its mmap files
            self._owners[key] = (j, weakref.ref(o), shadow)
            weakref.finalize(o, self.events.append, {"op": "release", "id": j})
        j, _, shadow = self._owners[key]
        r0, r1 = lo_hi
        flat = o.reshape(-1)[r0:r1]
        bits = np.uint16 if o.itemsize == 2 else np.uint32
        diff = np.flatnonzero(flat.view(bits) != shadow[r0:r1].view(bits))
        if diff.size:
            lo, hi = int(diff[0]), int(diff[-1]) + 1
            self.events.append({"op": "write", "id": j, "at": r0 + lo,
                                "data": self._store(flat[lo:hi])})
            shadow[r0 + lo:r0 + hi] = flat[lo:hi]
        return j

    def _arg(self, a, read_elems: int = -1):
        """An array argument: its contents, or (read_elems >= 0: the K / V
        arguments of gqa_attention, of which the call reads the first read_elems
        elements) its place in the manager's host array."""
        if read_elems >= 0 and isinstance(a, np.ndarray) and a.base is not None:
            o = _owner(a)
            if o is not a and o.flags["C_CONTIGUOUS"] and a.flags["C_CONTIGUOUS"]:
                off = a.ctypes.data - o.ctypes.data
                assert off % a.itemsize == 0
                at = off // a.itemsize
                j = self._sync_owner(o, (at, at + read_elems))
                return {"view": j, "at": at, "shape": list(a.shape)}
        return {"array": self._store(a)}

    # -- the module API the reference calls -------------------------------------
    def kv_cache_init(self, num_layers, max_seq_len, num_kv_heads, head_dim):
        self.events.append({"op": "call", "fn": "kv_cache_init",
                            "args": [int(num_layers), int(max_seq_len), int(num_kv_heads),
                                     int(head_dim)],
                            "raises": "RuntimeError" if self.fail_init else None})
        if self.fail_init:
            raise RuntimeError("injected: device allocation failed")
        self._pool = (np.zeros((num_layers, max_seq_len, num_kv_heads, head_dim), np.float16),
                      np.zeros((num_layers, max_seq_len, num_kv_heads, head_dim), np.float16))

    def kv_cache_free(self):
        self.events.append({"op": "call", "fn": "kv_cache_free", "args": []})
        self._pool = None

    def gqa_attention_cached(self, Q, K_new, V_new, Out, layer_idx, q_len, start_pos, num_heads,
                             num_kv_heads, head_dim, scale=0.0, causal=True):
        kp, vp = self._pool
        total = start_pos + q_len
        kp[layer_idx, start_pos:total] = K_new.reshape(q_len, num_kv_heads, head_dim)
        vp[layer_idx, start_pos:total] = V_new.reshape(q_len, num_kv_heads, head_dim)
        q = np.asarray(Q).reshape(q_len, num_heads, head_dim)
        exp = self.ref(q, kp[layer_idx, :total], vp[layer_idx, :total], start_pos, scale, causal)
        self.events.append({"op": "call", "fn": "gqa_attention_cached",
                            "args": [self._arg(Q), self._arg(K_new), self._arg(V_new),
                                     {"out": list(np.shape(Out)), "dtype": str(Out.dtype)},
                                     int(layer_idx), int(q_len), int(start_pos), int(num_heads),
                                     int(num_kv_heads), int(head_dim), float(scale),
                                     bool(causal)],
                            "expect": self._store(exp)})
        Out[...] = exp.reshape(Out.shape)

    def gqa_attention(self, Q, K, V, Out, q_len, kv_len, num_heads, num_kv_heads, head_dim,
                      start_pos=0, scale=0.0, causal=True):
        k = np.asarray(K).reshape(-1, num_kv_heads, head_dim)[:kv_len]
        v = np.asarray(V).reshape(-1, num_kv_heads, head_dim)[:kv_len]
        q = np.asarray(Q).reshape(q_len, num_heads, head_dim)
        exp = self.ref(q, k, v, start_pos, scale, causal)
        self.events.append({"op": "call", "fn": "gqa_attention",
                            "args": [self._arg(Q), self._arg(K, k.size), self._arg(V, v.size),
                                     {"out": list(np.shape(Out)), "dtype": str(Out.dtype)},
                                     int(q_len), int(kv_len), int(num_heads), int(num_kv_heads),
                                     int(head_dim), int(start_pos), float(scale), bool(causal)],
                            "expect": self._store(exp)})
        Out[...] = exp.reshape(Out.shape)

    def mark(self, text: str):
        """A note in the trace (what the recorded scenario does next)."""
        self.events.append({"op": "mark", "text": text})


def save(scenarios: dict, path: str = TRACE_FILE, meta: dict = None):
    """scenarios: name -> Recorder.  Arrays are stored once per distinct content
    (the three storage modes of one scenario carry the same inputs)."""
    import hashlib

    blob, names, index = {}, {}, {}
    for name, rec in scenarios.items():
        names[name] = {}
        for k, a in rec.arrays.items():
            h = hashlib.sha1(str(a.dtype).encode() + str(a.shape).encode() + a.tobytes())
            key = f"b{h.hexdigest()[:16]}"
            blob.setdefault(key, a)
            names[name][k] = key
        index[name] = rec.events
    blob["index"] = np.array(json.dumps({"scenarios": index, "names": names,
                                         "meta": meta or {}}))
    np.savez_compressed(path, **blob)


class Trace:
    """A loaded trace file: ``scenarios`` (name -> events), ``meta`` and the
    arrays the events name (``array(scenario, name)``)."""

    def __init__(self, path: str = TRACE_FILE):
        self.z = np.load(path)
        idx = json.loads(str(self.z["index"]))
        self.scenarios = idx["scenarios"]
        self.names = idx["names"]
        self.meta = idx["meta"]

    def array(self, scenario: str, name: str) -> np.ndarray:
        return self.z[self.names[scenario][name]]


def load(path: str = TRACE_FILE) -> Trace:
    return Trace(path)


class Replay:
    """Result of replaying one scenario: per attention call its output, the
    expected output, the call's arguments; per failed call the exception."""

    def __init__(self):
        self.calls = []     # (event, out or None, expect or None, exception or None)


def replay(trace: Trace, scenario: str, module, tmpdir: str = None,
           after_call=None) -> Replay:
    """Run the recorded events of ``scenario`` against ``module``."""
    events = trace.scenarios[scenario]
    hosts = {}          # id -> (flat ndarray, keep-alive objects)
    res = Replay()
    tmp = tempfile.TemporaryDirectory() if tmpdir is None else None
    base_dir = tmpdir or tmp.name
    try:
        for ev in events:
            op = ev["op"]
            if op == "host":
                dt = np.dtype(ev["dtype"])
                if ev["kind"] == "mmap":
                    path = os.path.join(base_dir, f"{scenario}_{ev['id']}.mmap")
                    fd = os.open(path, os.O_CREAT | os.O_EXCL | os.O_RDWR, 0o600)
                    try:
                        os.ftruncate(fd, ev["size"] * dt.itemsize)
                        mm = mmap.mmap(fd, ev["size"] * dt.itemsize, access=mmap.ACCESS_WRITE)
                    finally:
                        os.close(fd)
                    hosts[ev["id"]] = [np.frombuffer(mm, dtype=dt), mm, path]
                else:
                    hosts[ev["id"]] = [np.empty(ev["size"], dtype=dt), None, None]
            elif op == "write":
                flat = hosts[ev["id"]][0]
                data = trace.array(scenario, ev["data"])
                flat[ev["at"]:ev["at"] + data.size] = data
            elif op == "release":
                flat, mm, path = hosts.pop(ev["id"])
                del flat
                if mm is not None:
                    mm.close()
                    os.remove(path)
            elif op == "call":
                args, out = [], None
                for a in ev["args"]:
                    if isinstance(a, dict) and "view" in a:
                        flat = hosts[a["view"]][0]
                        n = int(np.prod(a["shape"]))
                        # the same kind of view the manager passes: a basic slice of
                        # its host array, reshaped (k_host[layer])
                        args.append(flat[a["at"]:a["at"] + n].reshape(a["shape"]))
                    elif isinstance(a, dict) and "array" in a:
                        args.append(np.array(trace.array(scenario, a["array"]), copy=True))
                    elif isinstance(a, dict) and "out" in a:
                        out = np.full(a["out"], np.nan, dtype=np.dtype(a["dtype"]))
                        args.append(out)
                    else:
                        args.append(a)
                exc = None
                try:
                    getattr(module, ev["fn"])(*args)
                except Exception as e:  # recorded as the call's outcome
                    exc = e
                expect = trace.array(scenario, ev["expect"]) if ev.get("expect") else None
                res.calls.append((ev, out, expect, exc))
                args = None  # no view outlives the call (a memory-mapped file closes later)
                if after_call is not None:
                    after_call(ev, out, exc)
        return res
    finally:
        for flat, mm, path in hosts.values():
            if mm is not None:
                del flat
                try:
                    mm.close()
                    os.remove(path)
                except (BufferError, OSError):
                    pass
        hosts.clear()
        if tmp is not None:
            tmp.cleanup()
