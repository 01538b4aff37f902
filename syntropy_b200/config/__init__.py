"""Layered configuration: defaults < TOML file < environment (SYN_<SECTION>_<KEY>) < CLI
overrides (section.key=value), with the origin of every value kept for diagnostics.
Reference: crates/config/src/{registry.rs,resolve.rs,validate.rs}; RFC-0054."""
from .schema import Config, load_config  # noqa: F401
