"""The ncu summary helpers of mxfp4_b200.profile (parsers run on CPU on ncu-format text)."""

from mxfp4_b200 import profile

LAUNCHES = '''==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","void mxb::gemm_tc_kernel<1, __nv_bfloat16>(CUtensorMap_st, mxb::TcOut, const unsigned char *, int, int, int, int)","1","7","(576, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","190.50"
"1","1","python","h","void mxb::gemm_tc_kernel<1, __nv_bfloat16>(CUtensorMap_st, mxb::TcOut, const unsigned char *, int, int, int, int)","1","7","(576, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","209.50"
"2","1","python","h","mxb::prepack_kernel(const unsigned char *)","1","7","(256, 1, 1)","(10, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","100,000"
'''

RAW = '''"ID","Kernel Name","gpu__time_duration.sum","dram__bytes_read.sum","launch__registers_per_thread"
"","","us","Mbyte","register/thread"
"0","gemm_tc_kernel<1, __nv_bfloat16>","186.24","50.63","96"
'''


def test_short_name():
    assert profile.short_name('void mxb::gemv_kernel<1, __nv_bfloat16>(const int *, int)') == \
        "mxb::gemv_kernel<1, __nv_bfloat16>"
    assert profile.short_name("mxb::prepack_kernel(const unsigned char *)") == "mxb::prepack_kernel"


def test_parse_launches_and_table():
    d = profile.parse_launches(LAUNCHES)
    assert d == {"mxb::gemm_tc_kernel<1, __nv_bfloat16>": [190500.0, 209500.0], "mxb::prepack_kernel": [100000.0]}
    t = profile.launch_table(d)
    assert "| mxb::gemm_tc_kernel<1, __nv_bfloat16> | 2 | 400.0 | 200.0 | 80.0 % |" in t
    assert "| mxb::prepack_kernel | 1 | 100.0 | 100.0 | 20.0 % |" in t


def test_parse_raw_and_table():
    launches = profile.parse_raw(RAW)
    assert len(launches) == 1 and launches[0]["gpu__time_duration.sum"] == "186.24 us"
    t = profile.raw_table(launches[0])
    assert "| DRAM read (`dram__bytes_read.sum`) | 50.63 Mbyte |" in t
    assert t.startswith("kernel: gemm_tc_kernel<1, __nv_bfloat16>")
