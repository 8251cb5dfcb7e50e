"""Drop-in for ``reaxv2/driver.py`` (``NativeInt8``).

The reference opens ``libcuda.so.1``, loads a cubin with ``cuModuleLoadData`` and keeps a function
cache (reaxv2/driver.py:3-13).  Here the kernels live in ``libreax_b200.so``; the constructor keeps the
reference's signature and attributes (``configs``, ``functions``, ``check``) and ignores the binary
path, because there is no cubin to load.
"""
from __future__ import annotations

from .. import _native


class NativeInt8:
    def __init__(self, binary=None, configs=None):
        self.configs = {} if configs is None else configs
        self.binary = binary
        self.cuda = _native.load()          # the C-ABI library takes the place of libcuda + module
        self.module = None
        self.functions = {}

    @staticmethod
    def check(status):
        """Non-zero status -> RuntimeError, with the library's message (reaxv2/driver.py:11-13)."""
        _native.check(status)
