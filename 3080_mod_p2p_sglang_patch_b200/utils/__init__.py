"""Timing, clock sampling, pre-flight checks, launch accounting and NVTX ranges."""
from . import nvtx  # noqa: F401
from .clocks import ClockSampler  # noqa: F401
from .preflight import preflight  # noqa: F401
from .timing import DeviceTimer, max_over_ranks  # noqa: F401
