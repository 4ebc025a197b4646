"""OpenAI-compatible HTTP API (FastAPI/uvicorn)."""
