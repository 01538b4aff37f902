"""Node daemon pieces: runner supervisor (restart with back-off, hang/stall detection) and
the runner lifecycle state machine (reference: crates/daemon, crates/runner)."""
from .supervisor import RunnerHealth, Supervisor, SupervisorConfig  # noqa: F401
from .lifecycle import Lifecycle, LifecycleState  # noqa: F401
