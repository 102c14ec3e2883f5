"""kernel_bench traffic: ncu's per-launch DRAM bytes grouped by GraphIR op and
set beside the cost model's logical bytes (the counterpart of the reference's
`llmi graph --json` cost fields, tools/modelconverter/GraphCommand.cpp:82-146).
Runs on a small hand-written CSV in ncu's --csv layout; no GPU needed."""
import argparse
import json

from llminfer_b200 import kernel_bench as KB

HEADER = ('"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream",'
          '"Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit",'
          '"Metric Value"')


def row(i, kernel, metric, unit, value):
    return (f'"{i}","1","python","h","{kernel}","1","7","(128, 1, 1)","(148, 1, 1)","0","10.0",'
            f'"Command line profiler metrics","{metric}","{unit}","{value}"')


def test_traffic_groups_launches_by_op_and_prices_them(tmp_path):
    lines = ["==PROF== Connected to process 1", HEADER]
    for call in range(2):
        base = 10 * call
        # ncu may print the names with their namespaces or without.
        partial = ("void llmi::decode::partial_rows<256, 4, 3>(llmi::decode::Args)" if call
                   else "void partial_rows<256, 4, 3>(Args)")
        merge = "llmi::decode::merge(llmi::decode::Args)" if call else "merge(Args)"
        lines += [row(base, partial, "dram__bytes_read.sum", "Gbyte", "1.07"),
                  row(base, partial, "dram__bytes_write.sum", "Mbyte", "3.5"),
                  row(base, partial, "gpu__time_duration.sum", "usecond", "155.0"),
                  row(base + 1, merge, "dram__bytes_read.sum", "Mbyte", "3.5"),
                  row(base + 1, merge, "dram__bytes_write.sum", "Mbyte", "0.5"),
                  row(base + 1, merge, "gpu__time_duration.sum", "usecond", "7.5")]
    path = tmp_path / "launches.csv"
    path.write_text("\n".join(lines) + "\n")
    args = argparse.Namespace(
        csv=str(path), workload="decode", batch=64, past=4096, capacity=8192,
        heads=[16, 4], dim=256, tokens=1)
    (line,) = KB.traffic(args)
    assert line["op"] == "CausalGqa" and line["calls"] == 2
    assert set(line["dispatches"]) == {"gqaScores", "gqaSoftmax"}
    assert line["dispatches"]["gqaScores"]["time_us_per_call"] == 155.0
    assert line["measured_dram_bytes_per_call"] == int(1.07e9 + 3.5e6 + 3.5e6 + 0.5e6)
    # CausalGqa logical bytes of 64 sequences at past 4096 (Cost.cpp:85-93):
    # q + K/V rows [0, 4097) + out.
    q = 16 * 256 * 2
    assert line["logical_bytes_per_call"] == 64 * (2 * q + 2 * 4097 * 4 * 256 * 2)
    assert 0.99 < line["measured_over_logical"] < 1.01
    json.dumps(line)
