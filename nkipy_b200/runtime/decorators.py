"""``baremetal_jit`` (reference ``runtime/decorators.py:10-64``).

Usable bare (``@baremetal_jit``) or with arguments; each call traces, plans
and runs the kernel on the B200 through ``baremetal_run_traced_kernel``.
"""

import functools

from nkipy_b200.runtime.compile import trace
from nkipy_b200.runtime.execute import baremetal_run_traced_kernel


def baremetal_jit(kernel_func=None, *, additional_compiler_args="", target=None):
    def decorator(func):
        @functools.wraps(func)
        def wrapper(*args, **kwargs):
            return baremetal_run_traced_kernel(
                trace(func), *args, additional_compiler_args=additional_compiler_args, target=target, **kwargs
            )

        return wrapper

    return decorator if kernel_func is None else decorator(kernel_func)
