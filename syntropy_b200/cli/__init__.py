"""Command line: ``python -m syntropy_b200 <command>`` (reference command tree:
crates/cli/src/args.rs:73-154)."""
