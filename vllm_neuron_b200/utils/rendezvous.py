"""Process-group rendezvous without a TCP port race.

The Trainium plugin patches torch's loopback TCPStore rendezvous because a port picked
free by the parent can be taken by another process before the store binds it
(``vllm/patches/port_hold_patch.py:1-16``).  Ranks that this framework spawns on one host
never need a port: they meet through a file store (``file://`` init method) in a private
temporary directory.  Multi-host launches keep ``env://`` (torchrun supplies MASTER_*).
"""

from __future__ import annotations

import os
import shutil
import tempfile

ENV = "VLLM_B200_INIT_METHOD"


class FileRendezvous:
    """A private ``file://`` init method for ranks spawned on this host; the directory is
    removed by :meth:`close` (or at interpreter exit via the context manager)."""

    def __init__(self):
        self.dir = tempfile.mkdtemp(prefix="vllm_b200_rdzv_")
        self.path = os.path.join(self.dir, "store")
        self.init_method = f"file://{self.path}"

    def export(self) -> str:
        """Publish the init method to child processes through the environment."""
        os.environ[ENV] = self.init_method
        return self.init_method

    def close(self) -> None:
        if os.environ.get(ENV) == self.init_method:
            os.environ.pop(ENV, None)
        shutil.rmtree(self.dir, ignore_errors=True)

    def __enter__(self) -> "FileRendezvous":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def init_method_from_env() -> str | None:
    return os.environ.get(ENV) or None
