"""thinksound.cpp_b200 — B200-native (sm_100a) MM-DiT hot path of thinksound.cpp.

The product is the C-ABI shared library ``libtsd_b200.so`` built from ``csrc/`` (declared in
``include/tsd.h``). This Python package is host-side plumbing over that C-ABI (ctypes), plus the
synthetic-weight/GGUF writer used by tests and the benchmark. The directory name contains a
dot, so load it with ``importlib`` under the module name ``tsd_b200`` (see ``load_package``
in ``__graft_entry__.py``).
"""
