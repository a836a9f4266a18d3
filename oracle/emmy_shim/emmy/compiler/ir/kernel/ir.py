from emmy._core import (  # noqa: F401
    Axis, BlockScaleLoad, CpAsyncCommit, CpAsyncCopy, CpAsyncWait, DataType, FragmentApply,
    FragmentPromote, FragmentRepack, FragmentRowReduce, KernelOp, LdmatrixLoad, MbarrierArrive,
    MbarrierArriveExpectTx, MbarrierInit, MbarrierWait, MmaSyncPtx, RegFragment, RegStore, Select,
    SelectBranch, SetMaxNReg, Smem, Sync, Tile, TmaDescriptor, TmaLoad, TreeHalve, WarpShuffle,
    WgmmaCommit, WgmmaDescriptor, WgmmaFence, WgmmaMma, WgmmaWait,
)
