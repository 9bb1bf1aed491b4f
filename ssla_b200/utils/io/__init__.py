"""Event-stream input (utils/io of the reference): .dat parsing on the host, payloads resident
in device memory, window slicing and batch collation on the GPU."""
from .dat_events_tools import (EV_STRING, EV_TYPE, EventStore, count_events, load_td_data, parse_header,
                               read_payload, write_dat)

__all__ = ["EV_STRING", "EV_TYPE", "EventStore", "count_events", "load_td_data", "parse_header", "read_payload",
           "write_dat"]
