"""Timing, clock sampling, pre-flight checks and launch accounting."""
from .clocks import ClockSampler  # noqa: F401
from .preflight import preflight  # noqa: F401
from .timing import DeviceTimer, max_over_ranks  # noqa: F401
