"""Per-backend op dispatch (reference: ``nkipy/core/ops/_registry.py:12-64``).

An ``Op`` holds one implementation per backend name; calling it runs the
implementation registered for ``get_backend()`` -- ``"hlo"`` while a kernel is
being traced, ``"cpu"`` otherwise -- and raises ``NotImplementedError`` naming
the available backends when there is none.
"""

from typing import Callable, Dict


class Op:
    def __init__(self, name: str):
        self.name = name
        self._impls: Dict[str, Callable] = {}

    def impl(self, backend: str) -> Callable:
        def register(fn: Callable) -> Callable:
            self._impls[backend] = fn
            return fn

        return register

    def __call__(self, *args, **kwargs):
        from nkipy_b200.core.backend import get_backend

        backend = get_backend()
        fn = self._impls.get(backend)
        if fn is None:
            have = ", ".join(self._impls) if self._impls else "none"
            raise NotImplementedError(
                f"Operation '{self.name}' not implemented for backend '{backend}'. Available backends: {have}"
            )
        return fn(*args, **kwargs)

    def __repr__(self) -> str:
        return f"Op('{self.name}', backends=[{', '.join(self._impls) or 'none'}])"
