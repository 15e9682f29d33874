"""Version of the API surface this package mirrors (rotalabs-accel's
``__version__``, src/rotalabs_accel/_version.py:3) and of this build."""

__version__ = "0.2.0"
__b200_version__ = "1.0.0"
