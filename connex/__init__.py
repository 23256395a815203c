"""connex: placeholder, filled in by the control-plane modules."""
__version__ = "0.2.1"
