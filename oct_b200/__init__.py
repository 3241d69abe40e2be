"""oct_b200 -- a B200-native (sm_100a) Prometheus reactor for Oct.

The product is ``libprometheus_reactor.so`` (C ABI v1, see include/prometheus_reactor.h),
built in-tree by :mod:`oct_b200.build`.  :mod:`oct_b200.reactor` is the host-side
binding that mirrors Oct's Go bridge.
"""
from .reactor import (  # noqa: F401
    ReactorIssue,
    Runtime,
    load_library,
    reduction_plan,
)

__all__ = ["ReactorIssue", "Runtime", "load_library", "reduction_plan"]
