"""Legacy shim (reference: core/model_loader.py:14): ``ModelManager`` keeps the
old load/generate entry points and forwards them to the engine factory."""

from b200serve.core.engine_factory import create_engine


class ModelManager:
    def __init__(self, config=None):
        self.engine = create_engine(config)

    def load(self, status_callback=None):
        self.engine.load(status_callback=status_callback)
        return self.engine

    def unload(self):
        self.engine.unload()

    @property
    def loaded(self) -> bool:
        return self.engine.is_loaded()

    def generate(self, messages, max_tokens=512, temperature=0.7, on_token=None, **kw):
        return self.engine.generate_streaming(messages, max_tokens, temperature, on_token=on_token, **kw)
