from attnrank.data.classes import EngineSettings, LayerScanSettings, ProfileSettings

__all__ = ["EngineSettings", "LayerScanSettings", "ProfileSettings"]
