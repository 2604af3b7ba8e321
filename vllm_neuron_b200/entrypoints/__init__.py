"""User entry points: OpenAI-compatible HTTP server and the ``vllm-b200`` CLI."""
