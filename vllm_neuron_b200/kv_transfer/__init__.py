"""Disaggregated prefill / decode: KV-cache transfer between serving engines."""

from .connector import HostStagedConnector, KVTransferError, make_connector  # noqa: F401
