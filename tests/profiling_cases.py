"""Raw Nsight counter cells and CSV logs for the reader's parity tests."""
from __future__ import annotations

import zlib

VALUES = ("0", "12", "-3", "1.5", ".25", "1e3", "2.5E-4", "1,234", "12,345,678.5", "1 234", "1 234", "1 234",
          "1,23", "12,34,567", "N/A", "", "  7  ", "inf", "nan", "1e400", "97.5%", "3.0 %", "(1, 2)", "0x10", True, None, 42, 3.5)
UNITS = ("", "byte", "Kbyte", "Mbyte", "Gbyte", "KB", "MiB", "GiB", "second", "msecond", "usecond", "us", "ns", "µs",
         "μsecond", "nanosecond", "cycle/second", "cycle/nsecond", "cycle/usecond", "GHz", "MHz", "%", "percent",
         "sector", "request", "inst", "instruction", "cycle", "count", "byte/second", "Kbyte/second", "Gbyte/s",
         "sector/s", "inst/second", "parsec", "byte/parsec", None, " byte ")
CELLS = [(v, u) for v in VALUES for u in UNITS
         if zlib.crc32(f"{v}|{u}".encode()) & 3 == 0 or u in ("byte", "%", "") or v in ("1,234", "N/A")]
CELLS = sorted(set(CELLS), key=lambda c: (str(c[0]), str(c[1])))

_HEADER = '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"'


def _row(launch, kernel, metric, unit, value):
    return f'"{launch}","4242","powerbench","box","{kernel}","1","7","(256, 1, 1)","(1184, 1, 1)","0","10.0","Command line profiler metrics","{metric}","{unit}","{value}"'


CSV_TEXTS = [
    "==PROF== Connected to process\n" + "\n".join([_HEADER,
        _row(0, "read_vector_kernel(...)", "dram__bytes_read.sum", "byte", "4,294,967,296"),
        _row(0, "read_vector_kernel(...)", "dram__bytes_write.sum", "Kbyte", "12.5"),
        _row(0, "read_vector_kernel(...)", "gpu__time_duration.sum", "usecond", "612.4"),
        _row(0, "read_vector_kernel(...)", "sm__cycles_elapsed.avg.per_second", "cycle/nsecond", "1.96"),
        _row(0, "read_vector_kernel(...)", "lts__t_sector_hit_rate.pct", "%", "0.4"),
        _row(0, "read_vector_kernel(...)", "l1tex__t_sectors_pipe_lsu_mem_local_op_ld.sum", "sector", "0"),
        _row(1, "tensor_mma_kernel<2>(...)", "sm__inst_executed_pipe_tensor.sum", "inst", "N/A"),
        _row(1, "tensor_mma_kernel<2>(...)", "gpu__time_duration.sum", "second", "0.0021")]) + "\n",
    "\n".join([_HEADER, _row(3, "sfu_kernel<0,false,4>", "smsp__inst_executed_pipe_sfu.sum", "inst", "1 048 576"),
               _row(3, "sfu_kernel<0,false,4>", "gpu__time_duration.sum", "msecond", "1,5")]),
    "no header here\n1,2,3\n",
    _HEADER + "\n",
]
