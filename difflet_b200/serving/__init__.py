"""OpenAI-compatible serving: engines (resident worker, replicas), HTTP API, video jobs."""
