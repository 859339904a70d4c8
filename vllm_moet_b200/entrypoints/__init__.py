"""User-facing entry points: the DeepSeek-V4-style chat encoding and the
OpenAI-compatible HTTP server."""
