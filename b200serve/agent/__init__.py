"""Agent layer above the engine: sandbox policy, tools, the multi-round agent loop.

It talks to the engine only through the BaseEngine contract (generate_streaming with
OpenAI ``tools``), so it runs on every backend name the factory resolves."""
