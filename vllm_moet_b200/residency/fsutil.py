"""Crash-safe file helpers shared by the pack stores and the planes cache."""
from __future__ import annotations

import contextlib
import fcntl
import json
import os
import time


def fsync_dir(path: str) -> None:
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def atomic_write_bytes(path: str, data: bytes) -> None:
    """Write to a unique temp file, fsync, rename over `path`, fsync the directory."""
    tmp = f"{path}.tmp.{os.getpid()}.{time.time_ns()}"
    try:
        with open(tmp, "xb") as f:
            f.write(data)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
        fsync_dir(os.path.dirname(os.path.abspath(path)))
    finally:
        with contextlib.suppress(FileNotFoundError):
            os.unlink(tmp)


def atomic_write_json(path: str, value: dict) -> None:
    atomic_write_bytes(path, json.dumps(value, sort_keys=True).encode())


def read_json(path: str):
    """-> parsed JSON, or None when missing or corrupt (callers rebuild)."""
    try:
        with open(path) as f:
            return json.load(f)
    except (FileNotFoundError, json.JSONDecodeError, UnicodeDecodeError, OSError):
        return None


@contextlib.contextmanager
def exclusive_lock(path: str):
    """flock(LOCK_EX) on a lock file next to the protected files."""
    fd = os.open(path, os.O_RDWR | os.O_CREAT | os.O_CLOEXEC, 0o644)
    try:
        fcntl.flock(fd, fcntl.LOCK_EX)
        yield
    finally:
        with contextlib.suppress(OSError):
            fcntl.flock(fd, fcntl.LOCK_UN)
        os.close(fd)
