"""HTTP serving surfaces: OpenAI-shaped (/v1/completions, /v1/chat/completions),
Anthropic-shaped (/v1/messages), native token-level generate (/v1/syntropy/generate, NDJSON)
and operational routes (/healthz, /readyz, /v1/models, /v1/syntropy/version, /metrics).
Reference route table: crates/api/src/routes.rs:51; native generate crates/api/src/native.rs."""
from .server import build_app  # noqa: F401
