"""OpenAI-compatible serving front end (HTTP app, engine driver thread, byte tokenizer, launcher)."""
