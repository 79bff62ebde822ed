"""``DeviceKernel`` (reference ``runtime/device_kernel.py:38-295``).

``compile_and_load`` keeps the reference's contract: trace, hash, plan once
per content hash (on-disk plan cache under ``build_dir/<name>_<hash>/``, plus
an in-process cache of loaded kernels); SPMD mode lets rank 0 plan and
broadcast the plan path (``dist.broadcast_object_list``) followed by a
barrier; MPMD mode plans per rank in ``rank_<r>`` sub-directories;
``cc_enabled`` / ``rank_id`` / ``world_size`` default from torch.distributed
and a collective kernel without them raises ``ValueError``.
"""

import atexit
import logging
import os
import shutil
import time
import types

from nkipy_b200.core.trace import NKIPyKernel
from nkipy_b200.runtime import compile as C
from nkipy_b200.runtime.device_tensor import DeviceTensor
from nkipy_b200.spike import SpikeModel

logger = logging.getLogger("nkipy_b200")

_LOADED_KERNELS = {}
atexit.register(_LOADED_KERNELS.clear)


def _dist():
    try:
        import torch.distributed as dist

        return dist
    except ImportError:  # pragma: no cover
        return None


def _is_distributed() -> bool:
    dist = _dist()
    return dist is not None and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


class DeviceKernel(SpikeModel):
    def __init__(self, model_ref, name, neff_path):
        super().__init__(model_ref, name, neff_path)

    @classmethod
    def compile_and_load(
        cls,
        kernel,
        *args,
        name=None,
        additional_compiler_args=None,
        use_cached_if_exists=True,
        build_dir=None,
        target=None,
        is_spmd=True,
        cc_enabled=None,
        rank_id=None,
        world_size=None,
        **kwargs,
    ):
        name = name or kernel.__name__
        distributed = _is_distributed()
        dist = _dist()
        if not is_spmd:
            rank = rank_id if rank_id is not None else (dist.get_rank() if distributed else None)
            compile_dir = os.path.join(build_dir or C.get_build_dir(), f"rank_{rank}") if rank is not None else build_dir
        else:
            compile_dir = build_dir
        resolved_cc = cc_enabled if cc_enabled is not None else distributed
        resolved_rank = rank_id if rank_id is not None else (dist.get_rank() if distributed else None)
        resolved_world = world_size if world_size is not None else (dist.get_world_size() if distributed else None)
        if resolved_cc and (resolved_rank is None or resolved_world is None):
            raise ValueError(
                "rank_id and world_size are required when cc_enabled=True and torch.distributed is not available "
                "for auto-detection"
            )
        plan_world = resolved_world if resolved_cc else 1

        if is_spmd and distributed:
            if dist.get_rank() == 0:
                info = list(cls._trace_and_compile(kernel, name, args, kwargs, use_cached_if_exists, compile_dir, plan_world, additional_compiler_args))
            else:
                info = [None, None]
            dist.broadcast_object_list(info, src=0)
            plan_path, cache_key = info
        else:
            plan_path, cache_key = cls._trace_and_compile(
                kernel, name, args, kwargs, use_cached_if_exists, compile_dir, plan_world, additional_compiler_args
            )

        if use_cached_if_exists and cache_key in _LOADED_KERNELS:
            return _LOADED_KERNELS[cache_key]
        if is_spmd and distributed:
            dist.barrier()
        if resolved_cc:
            k = cls.load_from_neff(plan_path, name=name, cc_enabled=True, rank_id=resolved_rank, world_size=resolved_world)
        else:
            k = cls.load_from_neff(plan_path, name=name)
        if use_cached_if_exists:
            _LOADED_KERNELS[cache_key] = k
        return k

    @classmethod
    def _trace_and_compile(cls, kernel, name, args, kwargs, use_cached_if_exists, build_dir, world, extra_args=None):
        if not isinstance(kernel, (types.FunctionType, NKIPyKernel)):
            raise NotImplementedError(f"Unsupported kernel type: {type(kernel)}")
        np_args = [a.numpy() if isinstance(a, DeviceTensor) else a for a in args]
        np_kwargs = {k: (v.numpy() if isinstance(v, DeviceTensor) else v) for k, v in kwargs.items()}
        traced, graph = C.specialize(kernel, np_args, np_kwargs)
        h = C.graph_hash(graph, world=world, extra=extra_args or "")
        cache_key = f"{name}_{h}"
        out_dir = os.path.join(build_dir or C.get_build_dir(), cache_key)
        plan_path = os.path.join(out_dir, f"{name}{C.PLAN_SUFFIX}")
        if use_cached_if_exists and os.path.exists(plan_path):
            logger.info("plan found in %s, using cached (hash=%s)", plan_path, h)
        else:
            if not use_cached_if_exists and os.path.exists(out_dir):
                shutil.rmtree(out_dir)
            t0 = time.time()
            C.compile_to_plan(traced, out_dir, name=name, world=world, use_cached_if_exists=False)
            logger.info("planned %s in %.3f s", name, time.time() - t0)
        return plan_path, cache_key
