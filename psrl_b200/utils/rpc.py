"""Minimal threaded RPC for the control plane (replaces Ray actor calls and the
gRPC/HTTP hops of the reference between router, PS and rollout replicas).

The server exposes named objects; each client connection gets a thread that
receives ``(target, method, args, kwargs)`` tuples and sends back
``("ok", result)`` or ``("err", message)``.  Transport is
``multiprocessing.connection`` over TCP on 127.0.0.1 with an auth key, so
tensors and dataclasses travel by pickling (CPU tensors through shared memory
with the ``file_system`` sharing strategy).
"""

from __future__ import annotations

import threading
import traceback
from multiprocessing.connection import Client, Listener

import torch.multiprocessing as tmp

# CPU tensors cross processes by shared-memory file name (no fd passing between
# unrelated processes); CUDA tensors are never sent through RPC (IPC handles are).
tmp.set_sharing_strategy("file_system")

DEFAULT_AUTHKEY = b"psrl_b200"


class RPCError(RuntimeError):
    pass


class RPCServer:
    def __init__(self, objects: dict, host: str = "127.0.0.1", port: int = 0, authkey: bytes = DEFAULT_AUTHKEY):
        self.objects = dict(objects)
        # a deep accept backlog: many ranks connect at once at start-up
        self.listener = Listener((host, port), backlog=128, authkey=authkey)
        self.address = self.listener.address
        self._stop = threading.Event()
        self._threads: list[threading.Thread] = []
        self._accept = threading.Thread(target=self._accept_loop, daemon=True, name="rpc-accept")
        self._accept.start()

    def register(self, name: str, obj) -> None:
        self.objects[name] = obj

    def _accept_loop(self):
        import multiprocessing
        while not self._stop.is_set():
            try:
                conn = self.listener.accept()
            except (OSError, EOFError, multiprocessing.AuthenticationError):
                if self._stop.is_set():
                    break
                continue          # a failed handshake must not stop the server
            t = threading.Thread(target=self._serve, args=(conn,), daemon=True, name="rpc-conn")
            t.start()
            self._threads.append(t)

    def _serve(self, conn):
        while not self._stop.is_set():
            try:
                msg = conn.recv()
            except (EOFError, OSError):
                break
            target, method, args, kwargs = msg
            try:
                fn = getattr(self.objects[target], method)
                res = ("ok", fn(*args, **kwargs))
            except Exception as exc:  # report to the caller, keep serving
                res = ("err", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()}")
            try:
                conn.send(res)
            except (OSError, EOFError):
                break
        conn.close()

    def close(self):
        self._stop.set()
        try:
            self.listener.close()
        except OSError:
            pass


def _connect_with_timeout(address, authkey: bytes, timeout: float):
    """``multiprocessing.connection.Client`` with a bounded connect + handshake.

    The socket stays in blocking mode; kernel receive/send timeouts bound the
    handshake and are cleared once it succeeded.
    """
    import socket
    import struct
    from multiprocessing.connection import Connection, answer_challenge, deliver_challenge

    sock = socket.create_connection(address, timeout=timeout)
    sock.settimeout(None)
    tv = struct.pack("ll", int(timeout), 0)
    sock.setsockopt(socket.SOL_SOCKET, socket.SO_RCVTIMEO, tv)
    sock.setsockopt(socket.SOL_SOCKET, socket.SO_SNDTIMEO, tv)
    conn = Connection(sock.detach())
    try:
        answer_challenge(conn, authkey)
        deliver_challenge(conn, authkey)
    except BlockingIOError as exc:
        conn.close()
        raise TimeoutError(f"RPC handshake with {address} timed out") from exc
    except BaseException:
        conn.close()
        raise
    s2 = socket.socket(fileno=conn.fileno())
    zero = struct.pack("ll", 0, 0)
    s2.setsockopt(socket.SOL_SOCKET, socket.SO_RCVTIMEO, zero)
    s2.setsockopt(socket.SOL_SOCKET, socket.SO_SNDTIMEO, zero)
    s2.detach()
    return conn


class RPCClient:
    def __init__(self, address, authkey: bytes = DEFAULT_AUTHKEY, retries: int = 600, timeout: float = 900.0):
        import time
        self.timeout = timeout
        last = None
        for _ in range(retries):
            try:
                self.conn = _connect_with_timeout(address, authkey, 30.0)
                break
            except (ConnectionRefusedError, OSError, EOFError, TimeoutError) as exc:
                last = exc
                time.sleep(0.1)
        else:
            raise RPCError(f"cannot connect to {address}: {last}")
        self._lock = threading.Lock()

    def call(self, target: str, method: str, *args, **kwargs):
        with self._lock:
            self.conn.send((target, method, args, kwargs))
            if not self.conn.poll(self.timeout):
                raise RPCError(f"RPC {target}.{method} got no reply within {self.timeout}s")
            status, val = self.conn.recv()
        if status != "ok":
            raise RPCError(val)
        return val

    def proxy(self, target: str) -> "_Proxy":
        return _Proxy(self, target)

    def close(self):
        try:
            self.conn.close()
        except OSError:
            pass


class _Proxy:
    def __init__(self, client: RPCClient, target: str):
        self._c = client
        self._t = target

    def __getattr__(self, name):
        def call(*a, **k):
            return self._c.call(self._t, name, *a, **k)
        return call
