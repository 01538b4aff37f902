"""Cluster control state: a hash-chained event log and a pure `apply` that folds events
into ClusterState (members, instances, plan epochs).  Single-box deployments run one
coordinator; the log makes state changes replayable and auditable.
Reference: crates/cluster/src/log/{entry.rs,event.rs,state.rs:35-248}."""
from .log import ClusterState, Event, EventLog, apply  # noqa: F401
