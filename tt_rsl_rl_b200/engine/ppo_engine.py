"""Placeholder replaced below."""


class PPOEngine:
    @staticmethod
    def unsupported_reason(alg):
        return "engine not built"

    @staticmethod
    def supports_models(actor, critic, alg_cfg):
        return "engine not built"
